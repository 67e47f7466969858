// Fused Adam step over the packed parameter vector [MLP weights | hash-grid table].
//
// Replaces adam_step_kernel / step_optimizer (ngp.train.cu:1261-1280, 1973-1980): gradient /
// loss scale; hash-grid entries whose gradient is exactly zero are skipped (sparse Adam with
// per-parameter step counters); MLP weights get L2 regularisation 1e-6; bias-corrected step;
// fp32 master weights and their fp16 copy are both written.
//
// B200 layout: four parameters per thread with 16-byte vector loads/stores, the gradient is
// fp32 (the library accumulates gradients in fp32), and the hash-grid part of the gradient is
// cleared in the same pass, so the next step's backward can accumulate into it without a
// separate memset.  Memory-bound: ~38 bytes per touched parameter, 16 per untouched one.
#include "common.cuh"

namespace ngp {
namespace {

struct AdamParams {
    uint32_t n_params;
    uint32_t n_mlp;  // parameters [0, n_mlp) are dense (MLP), the rest sparse (grid)
    float lr, beta1, beta2, eps, l2, inv_loss_scale;
    float* master;
    __half* params;
    float* grad;          // fp32 gradients, or
    const __half* grad16; // fp16 gradients (the reference's format; never cleared)
    float* m;
    float* v;
    uint32_t* steps;
    int clear_grid_grad;
    const float* lr_table;  // optional: lr_table[t] = bias-corrected rate after t steps, t <= table_len
    uint32_t table_len;
    uint32_t first;  // index of element 0 in the packed vector (a shard of it; a multiple of 4)
};

// Bias-corrected learning rate after `step` steps (ngp.train.cu:1275).
__device__ __forceinline__ float corrected_lr(float lr, float beta1, float beta2, uint32_t step) {
    return lr * sqrtf(1.0f - powf(beta2, static_cast<float>(step))) / (1.0f - powf(beta1, static_cast<float>(step)));
}

__device__ __forceinline__ void adam_one(const AdamParams& p, uint32_t i, float& master, float graw, float& m, float& v, uint32_t& step,
                                         __half& out) {
    float g          = graw * p.inv_loss_scale;
    const bool dense = p.first + i < p.n_mlp;
    if (!dense && g == 0.0f) return;
    const float w = master;
    if (dense) g = __fmaf_rn(p.l2, w, g);
    m = __fmaf_rn(p.beta1, m, (1.0f - p.beta1) * g);
    v = __fmaf_rn(p.beta2, v, (1.0f - p.beta2) * (g * g));
    step += 1u;
    // the rate depends only on the step count: read it from the table (the same function
    // evaluated once per step count) instead of two powf per parameter
    const float lr_t = step <= p.table_len ? __ldg(p.lr_table + step) : corrected_lr(p.lr, p.beta1, p.beta2, step);
    master           = w - lr_t * m / (sqrtf(v) + p.eps);
    out              = __float2half_rn(master);
}

template <bool HALF_GRAD>
__device__ __forceinline__ float4 load_grad4(const AdamParams& p, uint32_t q) {
    if constexpr (HALF_GRAD) {
        const uint2 raw  = reinterpret_cast<const uint2*>(p.grad16)[q];
        const float2 lo  = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
        const float2 hi  = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
        return make_float4(lo.x, lo.y, hi.x, hi.y);
    } else {
        return reinterpret_cast<const float4*>(p.grad)[q];
    }
}

template <bool HALF_GRAD>
__global__ void __launch_bounds__(256) adam_kernel(const __grid_constant__ AdamParams p) {
    const uint32_t q  = blockIdx.x * blockDim.x + threadIdx.x;  // group of 4
    const uint32_t i0 = q * 4u;
    if (i0 >= p.n_params) return;
    if (i0 + 4u <= p.n_params) {
        const float4 g  = load_grad4<HALF_GRAD>(p, q);
        const bool grid = p.first + i0 >= p.n_mlp;
        if (grid && g.x == 0.0f && g.y == 0.0f && g.z == 0.0f && g.w == 0.0f) return;  // untouched entries: one 16-byte read
        float4 w  = reinterpret_cast<float4*>(p.master)[q];
        float4 m  = reinterpret_cast<float4*>(p.m)[q];
        float4 v  = reinterpret_cast<float4*>(p.v)[q];
        uint4 s   = reinterpret_cast<uint4*>(p.steps)[q];
        uint2 hv  = reinterpret_cast<uint2*>(p.params)[q];
        __half* h = reinterpret_cast<__half*>(&hv);
        adam_one(p, i0 + 0u, w.x, g.x, m.x, v.x, s.x, h[0]);
        adam_one(p, i0 + 1u, w.y, g.y, m.y, v.y, s.y, h[1]);
        adam_one(p, i0 + 2u, w.z, g.z, m.z, v.z, s.z, h[2]);
        adam_one(p, i0 + 3u, w.w, g.w, m.w, v.w, s.w, h[3]);
        reinterpret_cast<float4*>(p.master)[q] = w;
        reinterpret_cast<float4*>(p.m)[q]      = m;
        reinterpret_cast<float4*>(p.v)[q]      = v;
        reinterpret_cast<uint4*>(p.steps)[q]   = s;
        reinterpret_cast<uint2*>(p.params)[q]  = hv;
        if (!HALF_GRAD && grid && p.clear_grid_grad) reinterpret_cast<float4*>(p.grad)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    for (uint32_t i = i0; i < p.n_params; ++i) {
        const float g = HALF_GRAD ? __half2float(p.grad16[i]) : p.grad[i];
        adam_one(p, i, p.master[i], g, p.m[i], p.v[i], p.steps[i], p.params[i]);
        if (!HALF_GRAD && p.first + i >= p.n_mlp && p.clear_grid_grad) p.grad[i] = 0.0f;
    }
}

__global__ void lr_table_kernel(float* __restrict__ table, uint32_t first, uint32_t count, float lr, float beta1, float beta2) {
    const uint32_t k = blockIdx.x * blockDim.x + threadIdx.x;
    if (k < count) table[first + k] = corrected_lr(lr, beta1, beta2, first + k);
}

int adam_launch(uint32_t n_params, uint32_t n_mlp, float lr, float beta1, float beta2, float eps, float l2_reg, float loss_scale,
                float* params_full_precision, uint16_t* params, float* gradients, const uint16_t* gradients16, float* first_moments,
                float* second_moments, uint32_t* param_steps, int clear_grid_gradients, const float* lr_table, uint32_t table_len, void* stream,
                uint32_t first = 0) {
    if (n_params == 0) return NGP_OK;
    if (first % 4u != 0) return fail(NGP_ERR_INVALID, "adam: the first index of a range must be a multiple of 4");
    if (params_full_precision == nullptr || params == nullptr || (gradients == nullptr) == (gradients16 == nullptr) || first_moments == nullptr ||
        second_moments == nullptr || param_steps == nullptr || (first == 0 && n_mlp > n_params) || n_mlp % 4u != 0 || loss_scale == 0.0f ||
        (table_len > 0 && lr_table == nullptr))
        return fail(NGP_ERR_INVALID, "adam: invalid input");
    if ((reinterpret_cast<uintptr_t>(params_full_precision) | reinterpret_cast<uintptr_t>(gradients) | reinterpret_cast<uintptr_t>(first_moments) |
         reinterpret_cast<uintptr_t>(second_moments) | reinterpret_cast<uintptr_t>(param_steps)) % 16u != 0 ||
        (reinterpret_cast<uintptr_t>(params) | reinterpret_cast<uintptr_t>(gradients16)) % 8u != 0)
        return fail(NGP_ERR_INVALID, "adam: buffers must be 16-byte aligned (fp16 buffers 8-byte)");
    AdamParams p{n_params,      n_mlp,     lr,       beta1,    beta2,       eps,
                 l2_reg,        1.0f / loss_scale, params_full_precision, reinterpret_cast<__half*>(params), gradients,
                 reinterpret_cast<const __half*>(gradients16), first_moments, second_moments, param_steps, clear_grid_gradients, lr_table, table_len,
                 first};
    const uint32_t groups = (n_params + 3u) / 4u;
    if (gradients16 != nullptr)
        adam_kernel<true><<<(groups + 255u) / 256u, 256, 0, as_stream(stream)>>>(p);
    else
        adam_kernel<false><<<(groups + 255u) / 256u, 256, 0, as_stream(stream)>>>(p);
    return check_launch("adam_kernel");
}

// Eight gradients per thread: two 16-byte fp32 loads, one 16-byte fp16 store and (clear) two
// 16-byte zero stores; the tail of n past a multiple of 8 one by one.
__global__ void grad_to_half_kernel(uint32_t n, float* __restrict__ src, __half* __restrict__ dst, int clear) {
    const uint32_t q = blockIdx.x * blockDim.x + threadIdx.x;  // group of 8
    const uint32_t i = q * 8u;
    if (i >= n) return;
    if (i + 8u <= n) {
        const float4 a = reinterpret_cast<const float4*>(src)[2u * q], b = reinterpret_cast<const float4*>(src)[2u * q + 1u];
        const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w), h2 = __floats2half2_rn(b.x, b.y),
                      h3 = __floats2half2_rn(b.z, b.w);
        reinterpret_cast<uint4*>(dst)[q] = make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                                                      *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
        if (clear) {
            reinterpret_cast<float4*>(src)[2u * q]      = make_float4(0.f, 0.f, 0.f, 0.f);
            reinterpret_cast<float4*>(src)[2u * q + 1u] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        return;
    }
    for (uint32_t k = i; k < n; ++k) {
        dst[k] = __float2half_rn(src[k]);
        if (clear) src[k] = 0.0f;
    }
}


// ---------------------------------------------------------------------------------------------
// Gradient reduce-scatter + Adam + parameter all-gather in one kernel over NVLink peer memory
// (the data-parallel hook between backward_network and step_optimizer, ngp.train.cpp:123-124).
// ---------------------------------------------------------------------------------------------
constexpr uint32_t kExchangeThreads = 256;
constexpr uint32_t kExchangeUnroll  = 8;  // ranks whose loads are unrolled (more: a loop)
constexpr uint64_t kExchangeWaitNs  = 2000000000ull;  // 2 s per cross-GPU wait, then an error status

__device__ __forceinline__ void store_release_sys(uint32_t* addr, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* addr) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits (one thread) until flags[base + q] >= epoch for every rank q; false after the time bound.
__device__ bool wait_all_ranks(const uint32_t* flags, uint32_t base, uint32_t world, uint32_t epoch) {
    const uint64_t start = now_ns();
    for (uint32_t q = 0; q < world; ++q) {
        while (static_cast<int32_t>(load_acquire_sys(flags + base + q) - epoch) < 0) {
            if (now_ns() - start > kExchangeWaitNs) return false;
            __nanosleep(64);
        }
    }
    return true;
}

__global__ void __launch_bounds__(kExchangeThreads) peer_exchange_adam_kernel(const __grid_constant__ PeerExchangeArgs a) {
    uint32_t* mine = a.flags[a.rank];
    __shared__ int s_ok;
    // arrival: this rank's gradients are complete (the conversion kernel ran before this one)
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        __threadfence_system();
        for (uint32_t q = 0; q < a.world; ++q) store_release_sys(a.flags[q] + a.rank, a.epoch);
    }
    if (threadIdx.x == 0) {
        s_ok = wait_all_ranks(mine, 0, a.world, a.epoch);
        if (!s_ok) atomicOr(a.status, 1u);
    }
    __syncthreads();
    if (s_ok) {
        AdamParams p{};
        p.n_mlp = a.n_mlp, p.lr = a.lr, p.beta1 = a.beta1, p.beta2 = a.beta2, p.eps = a.eps, p.l2 = a.l2;
        p.inv_loss_scale = 1.0f / a.loss_scale, p.lr_table = a.lr_table, p.table_len = a.table_len, p.first = 0;
        const uint32_t first = a.rank * a.shard;
        const uint32_t end   = min(first + a.shard, a.n_params);
        // eight parameters per thread and iteration: one 16-byte load per rank, all ranks' loads
        // in flight before the (rank-ordered) sum
        for (uint32_t i0 = first + (blockIdx.x * kExchangeThreads + threadIdx.x) * 8u; i0 < end; i0 += gridDim.x * kExchangeThreads * 8u) {
            float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            auto add = [&](const uint4& raw) {
                const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
                for (uint32_t k = 0; k < 4; ++k) {
                    const float2 f = __half22float2(h[k]);
                    g[2 * k] += f.x, g[2 * k + 1] += f.y;
                }
            };
            if (a.world <= kExchangeUnroll) {
                uint4 raw[kExchangeUnroll];
#pragma unroll
                for (uint32_t q = 0; q < kExchangeUnroll; ++q)
                    if (q < a.world) raw[q] = __ldcg(reinterpret_cast<const uint4*>(a.grads[q] + i0));
#pragma unroll
                for (uint32_t q = 0; q < kExchangeUnroll; ++q)
                    if (q < a.world) add(raw[q]);
            } else {
                for (uint32_t q = 0; q < a.world; ++q) add(__ldcg(reinterpret_cast<const uint4*>(a.grads[q] + i0)));
            }
            const bool grid = i0 >= a.n_mlp;
            bool zero       = true;
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k) zero = zero && g[k] == 0.0f;
            if (grid && zero) continue;  // untouched: params unchanged everywhere
            uint4 hv  = *reinterpret_cast<const uint4*>(a.params[a.rank] + i0);
            __half* h = reinterpret_cast<__half*>(&hv);
            if (i0 + 8u <= end) {
                float4* w4 = reinterpret_cast<float4*>(a.master + i0);
                float4* m4 = reinterpret_cast<float4*>(a.m + i0);
                float4* v4 = reinterpret_cast<float4*>(a.v + i0);
                uint4* s4  = reinterpret_cast<uint4*>(a.steps + i0);
                float4 w[2] = {w4[0], w4[1]}, m[2] = {m4[0], m4[1]}, v[2] = {v4[0], v4[1]};
                uint4 st[2] = {s4[0], s4[1]};
#pragma unroll
                for (uint32_t k = 0; k < 2; ++k) {
                    adam_one(p, i0 + 4u * k + 0u, w[k].x, g[4 * k + 0], m[k].x, v[k].x, st[k].x, h[4 * k + 0]);
                    adam_one(p, i0 + 4u * k + 1u, w[k].y, g[4 * k + 1], m[k].y, v[k].y, st[k].y, h[4 * k + 1]);
                    adam_one(p, i0 + 4u * k + 2u, w[k].z, g[4 * k + 2], m[k].z, v[k].z, st[k].z, h[4 * k + 2]);
                    adam_one(p, i0 + 4u * k + 3u, w[k].w, g[4 * k + 3], m[k].w, v[k].w, st[k].w, h[4 * k + 3]);
                }
                w4[0] = w[0], w4[1] = w[1], m4[0] = m[0], m4[1] = m[1], v4[0] = v[0], v4[1] = v[1], s4[0] = st[0], s4[1] = st[1];
            } else {
#pragma unroll
                for (uint32_t k = 0; k < 8; ++k)
                    if (i0 + k < end) adam_one(p, i0 + k, a.master[i0 + k], g[k], a.m[i0 + k], a.v[i0 + k], a.steps[i0 + k], h[k]);
            }
            // all-gather: the new parameters go to every rank's buffer
            for (uint32_t q = 0; q < a.world; ++q) *reinterpret_cast<uint4*>(a.params[q] + i0) = hv;
        }
    }
    // completion: after every CTA's writes, the last CTA tells every rank and waits for them all
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const uint32_t done = atomicAdd(mine + 2u * a.world, 1u);
        if (done == gridDim.x - 1u) {
            mine[2u * a.world] = 0u;
            __threadfence_system();
            for (uint32_t q = 0; q < a.world; ++q) store_release_sys(a.flags[q] + a.world + a.rank, a.epoch);
            if (!wait_all_ranks(mine, a.world, a.world, a.epoch)) atomicOr(a.status, 2u);
        }
    }
}
}  // namespace

int peer_exchange_adam(const PeerExchangeArgs& a, cudaStream_t stream) {
    const uint32_t groups = (a.shard + 7u) / 8u;
    uint32_t ctas         = (groups + kExchangeThreads - 1u) / kExchangeThreads;
    const uint32_t cap    = static_cast<uint32_t>(sm_count()) * 2u;  // two resident CTAs per SM (102 registers a thread)
    ctas                  = ctas < 1u ? 1u : (ctas > cap ? cap : ctas);
    peer_exchange_adam_kernel<<<ctas, kExchangeThreads, 0, stream>>>(a);
    return check_launch("peer_exchange_adam_kernel");
}

}  // namespace ngp

using namespace ngp;

extern "C" int ngp_adam_step(uint32_t n_params, uint32_t n_mlp, float lr, float beta1, float beta2, float eps, float l2_reg, float loss_scale,
                             float* params_full_precision, uint16_t* params, float* gradients, float* first_moments, float* second_moments,
                             uint32_t* param_steps, int clear_grid_gradients, void* stream) {
    clear_error();
    return adam_launch(n_params, n_mlp, lr, beta1, beta2, eps, l2_reg, loss_scale, params_full_precision, params, gradients, nullptr,
                       first_moments, second_moments, param_steps, clear_grid_gradients, nullptr, 0u, stream);
}

extern "C" int ngp_adam_lr_table(float* table, uint32_t first, uint32_t count, float lr, float beta1, float beta2, void* stream) {
    clear_error();
    if (count == 0) return NGP_OK;
    if (table == nullptr) return fail(NGP_ERR_INVALID, "adam lr table: null table");
    lr_table_kernel<<<(count + 255u) / 256u, 256, 0, as_stream(stream)>>>(table, first, count, lr, beta1, beta2);
    return check_launch("lr_table_kernel");
}

extern "C" int ngp_adam_step_table(uint32_t n_params, uint32_t n_mlp, float lr, float beta1, float beta2, float eps, float l2_reg,
                                   float loss_scale, float* params_full_precision, uint16_t* params, float* gradients, float* first_moments,
                                   float* second_moments, uint32_t* param_steps, int clear_grid_gradients, const float* lr_table,
                                   uint32_t table_len, void* stream) {
    clear_error();
    return adam_launch(n_params, n_mlp, lr, beta1, beta2, eps, l2_reg, loss_scale, params_full_precision, params, gradients, nullptr,
                       first_moments, second_moments, param_steps, clear_grid_gradients, lr_table, table_len, stream);
}

extern "C" int ngp_adam_step_f16(uint32_t n_params, uint32_t n_mlp, float lr, float beta1, float beta2, float eps, float l2_reg, float loss_scale,
                                 float* params_full_precision, uint16_t* params, const uint16_t* gradients, float* first_moments,
                                 float* second_moments, uint32_t* param_steps, const float* lr_table, uint32_t table_len, void* stream) {
    clear_error();
    if (gradients == nullptr) return fail(NGP_ERR_INVALID, "adam: null gradients");
    return adam_launch(n_params, n_mlp, lr, beta1, beta2, eps, l2_reg, loss_scale, params_full_precision, params, nullptr, gradients,
                       first_moments, second_moments, param_steps, 0, lr_table, table_len, stream);
}

extern "C" int ngp_adam_step_f16_range(uint32_t count, uint32_t first, uint32_t n_mlp, float lr, float beta1, float beta2, float eps, float l2_reg,
                                       float loss_scale, float* params_full_precision, uint16_t* params, const uint16_t* gradients,
                                       float* first_moments, float* second_moments, uint32_t* param_steps, const float* lr_table,
                                       uint32_t table_len, void* stream) {
    clear_error();
    if (gradients == nullptr) return fail(NGP_ERR_INVALID, "adam: null gradients");
    return adam_launch(count, n_mlp, lr, beta1, beta2, eps, l2_reg, loss_scale, params_full_precision, params, nullptr, gradients, first_moments,
                       second_moments, param_steps, 0, lr_table, table_len, stream, first);
}

extern "C" int ngp_gradients_to_half(uint32_t n, float* gradients, uint16_t* out, int clear, void* stream) {
    clear_error();
    if (n == 0) return NGP_OK;
    if (gradients == nullptr || out == nullptr) return fail(NGP_ERR_INVALID, "gradients to half: null pointer");
    if ((reinterpret_cast<uintptr_t>(gradients) | reinterpret_cast<uintptr_t>(out)) % 16u != 0)
        return fail(NGP_ERR_INVALID, "gradients to half: buffers must be 16-byte aligned");
    grad_to_half_kernel<<<(n + 8u * 256u - 1u) / (8u * 256u), 256, 0, as_stream(stream)>>>(n, gradients, reinterpret_cast<__half*>(out), clear);
    return check_launch("grad_to_half_kernel");
}
