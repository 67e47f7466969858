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

__global__ void grad_to_half_kernel(uint32_t n, float* __restrict__ src, __half* __restrict__ dst, int clear) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    dst[i] = __float2half_rn(src[i]);
    if (clear) src[i] = 0.0f;
}

}  // namespace
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
    grad_to_half_kernel<<<(n + 255u) / 256u, 256, 0, as_stream(stream)>>>(n, gradients, reinterpret_cast<__half*>(out), clear);
    return check_launch("grad_to_half_kernel");
}
