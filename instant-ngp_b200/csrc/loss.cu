// Volume compositing, training loss, analytic compositing backward and deterministic
// compaction of the training batch; evaluation compositing (PSNR / comparison image).
//
// Replaces K10-K13 (ngp.train.cu:669-874) and the host wrappers
// compute_training_loss_and_compact_samples / pad_compacted_training_batch (1932-1956).
//
// The reference reserves compacted slots with a global atomic (ray order nondeterministic) and
// composites each ray in one thread.  Here one warp composites one ray, 32 samples at a time:
// each lane recomputes its transmittance and colour prefix by a sequential loop over the
// earlier lanes' values (shuffled), in the same order as a one-thread loop, so results are
// identical to the sequential compositing while a ray's samples are processed in parallel.
// Pass 1 counts the samples each ray keeps (front-to-back until the transmittance drops below
// 1e-4), one CTA scans the per-CTA totals, and pass 2 writes each ray's compacted samples,
// network-output gradients and loss at its prefix offset.
#include <mutex>

#include "sampler.cuh"

namespace ngp {
namespace {

constexpr uint32_t kRaysPerCta = 8u;
constexpr uint32_t kCtaThreads = kRaysPerCta * 32u;
constexpr uint32_t kThreads    = 128u;  // evaluation compositing (one thread per pixel)

struct LossParams {
    uint32_t rays_per_batch;        // rays of the step (scales the loss and its gradient)
    uint32_t step;
    const uint32_t* ray_counter;    // optional: rays actually marched (<= rays_per_batch)
    const uint8_t* pixels;
    uint32_t frame_count, width, height;
    const __half* network_output;   // [samples][16]
    const uint32_t* ray_indices;    // optional: batch ray index of each marched ray
    const float* rays;              // [ray][6]
    uint32_t* numsteps;             // [ray][2]; rewritten with the compacted (count, base)
    const float* coords;            // pre-compaction sample records
    float* coords_out;              // compacted records [NETWORK_BATCH_SIZE][7]
    __half* dloss_doutput;          // [NETWORK_BATCH_SIZE][16]
    float* loss_output;             // [ray] (may be null)
    int loss_kind;                  // kLossL2 (the reference) or kLossHuber
    float4* ray_rgb;                // scratch [ray]: composited colour, pass 1 -> pass 2
    uint32_t* kept;                 // scratch [ray]: samples kept by compositing
    uint32_t* block_totals;         // scratch [ray blocks]
    uint32_t batch;                 // NETWORK_BATCH_SIZE
};

__device__ __forceinline__ uint32_t loss_rays(const LossParams& p) {
    const uint32_t n = p.ray_counter != nullptr ? *p.ray_counter : p.rays_per_batch;
    return min(n, p.rays_per_batch);
}

// Target pixel and random background of ray `ray_index` in this step (ngp.train.cu:781-796).
__device__ __forceinline__ void ray_target(uint32_t step, uint32_t rays_per_batch, const uint8_t* __restrict__ pixels, uint32_t frame_count,
                                           uint32_t width, uint32_t height, uint32_t ray_index, float3& bg, float3& target) {
    Pcg32 rng{kTrainSeed};
    rng.advance(static_cast<uint64_t>(step) << 32u);
    rng.advance(static_cast<uint64_t>(ray_index) * kRandPerRay);
    const uint32_t image = static_cast<uint32_t>((static_cast<uint64_t>(ray_index) * frame_count) / rays_per_batch) % frame_count;
    float u = rng.next_float(), v = rng.next_float();
    uint32_t px = min(static_cast<uint32_t>(u * static_cast<float>(width)), width - 1u);
    uint32_t py = min(static_cast<uint32_t>(v * static_cast<float>(height)), height - 1u);
    u           = (static_cast<float>(px) + 0.5f) / static_cast<float>(width);
    v           = (static_cast<float>(py) + 0.5f) / static_cast<float>(height);
    bg          = {rng.next_float(), rng.next_float(), rng.next_float()};
    px          = min(static_cast<uint32_t>(u * static_cast<float>(width)), width - 1u);
    py          = min(static_cast<uint32_t>(v * static_cast<float>(height)), height - 1u);
    const float4 texel = read_texel(px, py, image, width, height, pixels);
    const float3 bgl   = {srgb_to_linear_c(bg.x), srgb_to_linear_c(bg.y), srgb_to_linear_c(bg.z)};
    target = {linear_to_srgb_c(__fmaf_rn(1.0f - texel.w, bgl.x, texel.x)), linear_to_srgb_c(__fmaf_rn(1.0f - texel.w, bgl.y, texel.y)),
              linear_to_srgb_c(__fmaf_rn(1.0f - texel.w, bgl.z, texel.z))};
}

__device__ __forceinline__ void ray_target(const LossParams& p, uint32_t ray_index, float3& bg, float3& target) {
    ray_target(p.step, p.rays_per_batch, p.pixels, p.frame_count, p.width, p.height, ray_index, bg, target);
}

__device__ __forceinline__ void load_output(const __half* o, float& r, float& g, float& b, float& d) {
    const uint2 v    = *reinterpret_cast<const uint2*>(o);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
    const float2 rg = __half22float2(h[0]), bd = __half22float2(h[1]);
    r = rg.x, g = rg.y, b = bd.x, d = bd.y;
}

// Transmittance before this lane's sample: T * q_0 * q_1 * ... * q_{lane-1}, multiplied in lane
// order exactly as the sequential loop does.
// Only lanes below `count` (warp-uniform) get their value: the loop stops after lane count-2.
__device__ __forceinline__ float prefix_transmittance(float T, float q, uint32_t count) {
    const uint32_t lane = threadIdx.x & 31u;
    float Tb            = T;
#pragma unroll
    for (uint32_t k = 0; k < 31; ++k) {
        if (k + 1u >= count) break;
        const float qk = __shfl_sync(0xFFFFFFFFu, q, k);
        if (k < lane) Tb *= qk;
    }
    return Tb;
}

// Loss of a ray's composited colour against its target, per colour channel residual d.
//  L2 (the reference, ngp.train.cu:817-819): d^2, gradient 2 d.
//  Huber (the loss of the original instant-ngp NeRF, delta = 0.1, divided by 5 so that it equals
//  the L2 loss for residuals below delta): (|d| <= 0.1 ? 5 d^2 : |d| - 0.05) / 5, gradient
//  |d| <= 0.1 ? 2 d : sign(d) / 5.
enum : int { kLossL2 = 0, kLossHuber = 1 };

__device__ __forceinline__ float3 loss_gradient(float3 d, int kind) {
    if (kind == kLossHuber) {
        auto g = [](float v) { return fabsf(v) <= 0.1f ? 2.0f * v : copysignf(0.2f, v); };
        return {g(d.x), g(d.y), g(d.z)};
    }
    return {2.0f * d.x, 2.0f * d.y, 2.0f * d.z};
}

// Per-ray loss value: the mean over the 3 channels, divided by the ray count (ngp.train.cu:820).
__device__ __forceinline__ float loss_value(float3 d, int kind, uint32_t rays_per_batch) {
    if (kind == kLossHuber) {
        auto h = [](float v) { const float a = fabsf(v); return a <= 0.1f ? v * v : __fmaf_rn(a, 0.2f, -0.01f); };
        return (h(d.x) + h(d.y) + h(d.z)) / (3.0f * static_cast<float>(rays_per_batch));
    }
    return __fmaf_rn(d.z, d.z, __fmaf_rn(d.x, d.x, d.y * d.y)) / (3.0f * static_cast<float>(rays_per_batch));
}

// Gradients of one ray's first cn samples (rest of K11, ngp.train.cu:804-859): dL/d(raw rgb) and
// dL/d(raw density) per sample, times `scale`; the sample records are also copied to cout when
// it is not null.  The whole warp calls it for one ray.
__device__ __forceinline__ void ray_gradients(float3 rgb, float3 grad, float scale, const float* __restrict__ ray, const float* __restrict__ cin,
                                              const __half* __restrict__ out, float* __restrict__ cout, __half* __restrict__ dout, uint32_t cn) {
    const uint32_t lane = threadIdx.x & 31u;
    const float3 origin = {ray[0], ray[1], ray[2]};
    float T             = 1.0f;
    float3 acc          = {0.0f, 0.0f, 0.0f};
    for (uint32_t c0 = 0; c0 < cn; c0 += 32u) {
        const uint32_t j = c0 + lane;
        const bool valid = j < cn;
        float cv[7]      = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        float mr = 0.f, mg = 0.f, mb = 0.f, md = 0.f;
        if (valid) {
            const float* c = cin + static_cast<uint64_t>(j) * 7u;
#pragma unroll
            for (int q = 0; q < 7; ++q) cv[q] = c[q];
            if (cout != nullptr) {
                float* co = cout + static_cast<uint64_t>(j) * 7u;
#pragma unroll
                for (int q = 0; q < 7; ++q) co[q] = cv[q];
            }
            load_output(out + static_cast<uint64_t>(j) * 16u, mr, mg, mb, md);
        }
        const float dt     = cv[3];
        const float3 col   = {sigmoidf_(mr), sigmoidf_(mg), sigmoidf_(mb)};
        const float alpha  = valid ? 1.0f - __expf(-expf(md) * dt) : 0.0f;
        const uint32_t nv  = min(32u, cn - c0);
        const float Tb     = prefix_transmittance(T, 1.0f - alpha, nv);
        const float weight = alpha * Tb;
        // colour prefix including this sample, accumulated in sample order (lanes below nv)
        float3 a = acc;
        for (uint32_t q = 0; q < nv; ++q) {
            const float wq = __shfl_sync(0xFFFFFFFFu, weight, q);
            const float cx = __shfl_sync(0xFFFFFFFFu, col.x, q), cy = __shfl_sync(0xFFFFFFFFu, col.y, q), cz = __shfl_sync(0xFFFFFFFFu, col.z, q);
            if (q <= lane) {
                a.x = __fmaf_rn(wq, cx, a.x);
                a.y = __fmaf_rn(wq, cy, a.y);
                a.z = __fmaf_rn(wq, cz, a.z);
            }
        }
        const float Ta = Tb * (1.0f - alpha);
        if (valid) {
            const float depth   = norm3df(cv[0] - origin.x, cv[1] - origin.y, cv[2] - origin.z);
            const float3 suffix = {rgb.x - a.x, rgb.y - a.y, rgb.z - a.z};
            const float g0      = scale * (weight * grad.x * (col.x * (1.0f - col.x)));
            const float g1      = scale * (weight * grad.y * (col.y * (1.0f - col.y)));
            const float g2      = scale * (weight * grad.z * (col.z * (1.0f - col.z)));
            const float dd      = expf(fminf(fmaxf(md, -15.0f), 15.0f));
            const float sum = __fmaf_rn(grad.z, __fmaf_rn(Ta, col.z, -suffix.z),
                                        __fmaf_rn(grad.x, __fmaf_rn(Ta, col.x, -suffix.x), grad.y * __fmaf_rn(Ta, col.y, -suffix.y)));
            const float g3 = __fmaf_rn(scale, dd * (dt * sum), (md > -10.0f && depth < 0.1f) ? 1e-4f : 0.0f);
            uint4* d       = reinterpret_cast<uint4*>(dout + static_cast<uint64_t>(j) * 16u);
            __half2 h01 = __floats2half2_rn(g0, g1), h23 = __floats2half2_rn(g2, g3);
            d[0]        = make_uint4(*reinterpret_cast<uint32_t*>(&h01), *reinterpret_cast<uint32_t*>(&h23), 0u, 0u);
            d[1]        = make_uint4(0u, 0u, 0u, 0u);
        }
        const uint32_t last = min(31u, cn - 1u - c0);
        T                   = __shfl_sync(0xFFFFFFFFu, Ta, last);
        acc.x               = __shfl_sync(0xFFFFFFFFu, a.x, last);
        acc.y               = __shfl_sync(0xFFFFFFFFu, a.y, last);
        acc.z               = __shfl_sync(0xFFFFFFFFu, a.z, last);
    }
}

__global__ void __launch_bounds__(1024) scan_kept_kernel(uint32_t* __restrict__ totals, uint32_t n_blocks, uint32_t* __restrict__ compacted_counter,
                                                         uint32_t batch) {
    uint32_t carry = 0;
    for (uint32_t b = 0; b < n_blocks; b += 1024u) {
        const uint32_t k = b + threadIdx.x;
        const uint32_t v = k < n_blocks ? totals[k] : 0u;
        uint32_t sum;
        const uint32_t ex = block_exclusive_scan(v, sum);
        if (k < n_blocks) totals[k] = carry + ex;
        carry += sum;
    }
    if (threadIdx.x == 0) *compacted_counter = carry < batch ? carry : batch;
}


// Pass 1 (first loop of K11, ngp.train.cu:751-802): composite, count the kept samples.
__global__ void __launch_bounds__(kCtaThreads) loss_pass1_kernel(const __grid_constant__ LossParams p) {
    __shared__ uint32_t s_kept[kRaysPerCta];
    const uint32_t n    = loss_rays(p);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t i    = blockIdx.x * kRaysPerCta + warp;
    uint32_t kept       = 0;
    if (i < n) {
        const uint32_t steps = p.numsteps[2u * i], base = p.numsteps[2u * i + 1u];
        const __half* out    = p.network_output + static_cast<uint64_t>(base) * 16u;
        const float* c       = p.coords + static_cast<uint64_t>(base) * 7u;
        float T              = 1.0f;
        float3 rgb           = {0.0f, 0.0f, 0.0f};
        for (uint32_t c0 = 0; c0 < steps; c0 += 32u) {
            const uint32_t j = c0 + lane;
            const bool valid = j < steps;
            float r = 0.f, g = 0.f, b = 0.f, d = 0.f, dt = 0.f;
            if (valid) {
                load_output(out + static_cast<uint64_t>(j) * 16u, r, g, b, d);
                dt = c[static_cast<uint64_t>(j) * 7u + 3u];
            }
            const float alpha = valid ? 1.0f - __expf(-expf(d) * dt) : 0.0f;
            const float3 col  = {sigmoidf_(r), sigmoidf_(g), sigmoidf_(b)};
            const float Tb    = prefix_transmittance(T, 1.0f - alpha, min(32u, steps - c0));
            const bool keep   = valid && !(Tb < kTransmittanceEps);
            const uint32_t nk = __popc(__ballot_sync(0xFFFFFFFFu, keep));
            const float w     = alpha * Tb;
            for (uint32_t k = 0; k < nk; ++k) {
                const float wk = __shfl_sync(0xFFFFFFFFu, w, k);
                rgb.x          = __fmaf_rn(wk, __shfl_sync(0xFFFFFFFFu, col.x, k), rgb.x);
                rgb.y          = __fmaf_rn(wk, __shfl_sync(0xFFFFFFFFu, col.y, k), rgb.y);
                rgb.z          = __fmaf_rn(wk, __shfl_sync(0xFFFFFFFFu, col.z, k), rgb.z);
            }
            if (nk > 0) T = __shfl_sync(0xFFFFFFFFu, Tb * (1.0f - alpha), nk - 1u);
            kept += nk;
            if (nk < min(32u, steps - c0)) break;
        }
        if (kept == steps) {
            float3 bg, target;
            ray_target(p, p.ray_indices != nullptr ? p.ray_indices[i] : i, bg, target);
            rgb.x = __fmaf_rn(T, bg.x, rgb.x);
            rgb.y = __fmaf_rn(T, bg.y, rgb.y);
            rgb.z = __fmaf_rn(T, bg.z, rgb.z);
        }
        if (lane == 0) {
            p.ray_rgb[i] = make_float4(rgb.x, rgb.y, rgb.z, 0.0f);
            p.kept[i]    = kept;
        }
    }
    if (lane == 0) s_kept[warp] = kept;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t total = 0;
        for (uint32_t w = 0; w < kRaysPerCta; ++w) total += s_kept[w];
        p.block_totals[blockIdx.x] = total;
    }
}

// Pass 2 (rest of K11, ngp.train.cu:804-859): clamp to the batch, copy the kept samples, write
// dL/d(raw rgb) and dL/d(raw density) per sample, scaled by 128 / rays_per_batch.
__global__ void __launch_bounds__(kCtaThreads) loss_pass2_kernel(const __grid_constant__ LossParams p) {
    const uint32_t n    = loss_rays(p);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t i    = blockIdx.x * kRaysPerCta + warp;
    uint32_t cbase      = p.block_totals[blockIdx.x];
    for (uint32_t w = 0; w < warp; ++w) {
        const uint32_t q = blockIdx.x * kRaysPerCta + w;
        cbase += q < n ? p.kept[q] : 0u;
    }
    if (i >= n) return;
    const uint32_t k         = p.kept[i];
    const uint32_t remaining = cbase < p.batch ? p.batch - cbase : 0u;
    const uint32_t cn        = k < remaining ? k : remaining;
    const uint32_t base      = p.numsteps[2u * i + 1u];
    __syncwarp();
    if (lane == 0) {
        p.numsteps[2u * i]      = cn;
        p.numsteps[2u * i + 1u] = cbase;
    }
    if (cn == 0) return;

    float3 bg, target;
    ray_target(p, p.ray_indices != nullptr ? p.ray_indices[i] : i, bg, target);
    const float4 rr   = p.ray_rgb[i];
    const float3 rgb  = {rr.x, rr.y, rr.z};
    const float3 diff = {rgb.x - target.x, rgb.y - target.y, rgb.z - target.z};
    if (p.loss_output != nullptr && lane == 0) p.loss_output[i] = loss_value(diff, p.loss_kind, p.rays_per_batch);
    ray_gradients(rgb, loss_gradient(diff, p.loss_kind), kLossScale / static_cast<float>(p.rays_per_batch), p.rays + static_cast<uint64_t>(i) * 6u,
                  p.coords + static_cast<uint64_t>(base) * 7u, p.network_output + static_cast<uint64_t>(base) * 16u,
                  p.coords_out + static_cast<uint64_t>(cbase) * 7u, p.dloss_doutput + static_cast<uint64_t>(cbase) * 16u, cn);
}

// ---------------------------------------------------------------------------------------------
// Density-first flow.  Which samples a ray keeps depends only on the densities (the
// transmittance), so the pre-compaction pass needs only the density network; the colour
// network then runs on the kept samples alone.  The results are identical to the flow above:
// the kept set, its order and every network output are the same (each output row is a function
// of its own input row), so the composited colours, losses and gradients match bit for bit.
//   1. keep pass: per ray, the kept count from the raw densities (same transmittance loop);
//   2. one CTA scans the per-CTA totals;
//   3. copy pass: each ray whose compacted base lies inside the batch copies all its kept
//      samples (records and encoded positions) to the compacted buffers, which hold
//      kCompactedRows = batch + kMarchSteps rows, so the ray straddling the batch end is whole;
//   4. (the caller runs the full network on the compacted rows)
//   5. loss pass: composite each ray from its compacted outputs, then the gradients of its
//      samples inside the batch (as pass 2 above).
// ---------------------------------------------------------------------------------------------
static_assert(kCompactedRows == kNetworkBatch + kMarchSteps, "compacted rows");

struct KeepParams {
    uint32_t rays_per_batch;
    const uint32_t* ray_counter;
    const __half* density;      // [samples] raw density
    const float* coords;        // pre-compaction records
    const __half* enc;          // optional: [32][enc_stride] encoded positions
    uint32_t enc_stride;
    uint32_t* numsteps;         // [ray][2] (steps, base) in; (kept, compacted base) out
    float* coords_out;          // [kCompactedRows][7]
    __half* enc_out;            // optional: [32][kCompactedRows]
    uint32_t* kept;             // scratch [ray]
    uint32_t* steps;            // scratch [ray]: marched samples
    uint32_t* block_totals;     // scratch [ray blocks]
};

__device__ __forceinline__ uint32_t keep_rays(const KeepParams& p) {
    const uint32_t n = p.ray_counter != nullptr ? *p.ray_counter : p.rays_per_batch;
    return min(n, p.rays_per_batch);
}

// Step 1 (the transmittance part of pass 1).
__global__ void __launch_bounds__(kCtaThreads) keep_pass_kernel(const __grid_constant__ KeepParams p) {
    __shared__ uint32_t s_kept[kRaysPerCta];
    const uint32_t n    = keep_rays(p);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t i    = blockIdx.x * kRaysPerCta + warp;
    uint32_t kept       = 0;
    if (i < n) {
        const uint32_t steps = p.numsteps[2u * i], base = p.numsteps[2u * i + 1u];
        const __half* dens   = p.density + base;
        const float* c       = p.coords + static_cast<uint64_t>(base) * 7u;
        float T              = 1.0f;
        for (uint32_t c0 = 0; c0 < steps; c0 += 32u) {
            const uint32_t j  = c0 + lane;
            const bool valid  = j < steps;
            const float d     = valid ? __half2float(dens[j]) : 0.0f;
            const float dt    = valid ? c[static_cast<uint64_t>(j) * 7u + 3u] : 0.0f;
            const float alpha = valid ? 1.0f - __expf(-expf(d) * dt) : 0.0f;
            const float Tb    = prefix_transmittance(T, 1.0f - alpha, min(32u, steps - c0));
            const bool keep   = valid && !(Tb < kTransmittanceEps);
            const uint32_t nk = __popc(__ballot_sync(0xFFFFFFFFu, keep));
            if (nk > 0) T = __shfl_sync(0xFFFFFFFFu, Tb * (1.0f - alpha), nk - 1u);
            kept += nk;
            if (nk < min(32u, steps - c0)) break;
        }
        if (lane == 0) {
            p.kept[i]  = kept;
            p.steps[i] = steps;
        }
    }
    if (lane == 0) s_kept[warp] = kept;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t total = 0;
        for (uint32_t w = 0; w < kRaysPerCta; ++w) total += s_kept[w];
        p.block_totals[blockIdx.x] = total;
    }
}

// Step 3.
__global__ void __launch_bounds__(kCtaThreads) compact_copy_kernel(const __grid_constant__ KeepParams p) {
    const uint32_t n    = keep_rays(p);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t i    = blockIdx.x * kRaysPerCta + warp;
    uint32_t cbase      = p.block_totals[blockIdx.x];
    for (uint32_t w = 0; w < warp; ++w) {
        const uint32_t q = blockIdx.x * kRaysPerCta + w;
        cbase += q < n ? p.kept[q] : 0u;
    }
    if (i >= n) return;
    const uint32_t k    = cbase < kNetworkBatch ? p.kept[i] : 0u;
    const uint32_t base = p.numsteps[2u * i + 1u];
    __syncwarp();
    if (lane == 0) {
        p.numsteps[2u * i]      = k;
        p.numsteps[2u * i + 1u] = cbase;
    }
    const float* __restrict__ cin = p.coords + static_cast<uint64_t>(base) * 7u;
    float* __restrict__ cout      = p.coords_out + static_cast<uint64_t>(cbase) * 7u;
    for (uint32_t j = lane; j < k * 7u; j += 32u) cout[j] = __ldg(cin + j);
    if (p.enc_out != nullptr && rows_layout(p.enc_stride)) {
        // row-major encodings: a sample's 64-byte row is copied to its compacted row
        const uint4* __restrict__ src = reinterpret_cast<const uint4*>(p.enc) + static_cast<uint64_t>(base) * 4u;
        uint4* __restrict__ dst       = reinterpret_cast<uint4*>(p.enc_out) + static_cast<uint64_t>(cbase) * 4u;
        for (uint32_t j = lane; j < k * 4u; j += 32u) dst[j] = __ldg(src + j);
    } else if (p.enc_out != nullptr) {
        // all 32 features of a sample are loaded before any is stored (independent loads in flight)
        const unsigned short* __restrict__ src = reinterpret_cast<const unsigned short*>(p.enc) + base;
        unsigned short* __restrict__ dst       = reinterpret_cast<unsigned short*>(p.enc_out) + cbase;
        for (uint32_t j = lane; j < k; j += 32u) {
            unsigned short v[32];
#pragma unroll
            for (uint32_t f = 0; f < 32u; ++f) v[f] = __ldg(src + static_cast<uint64_t>(f) * p.enc_stride + j);
#pragma unroll
            for (uint32_t f = 0; f < 32u; ++f) dst[static_cast<uint64_t>(f) * kCompactedRows + j] = v[f];
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Progressive density evaluation.  A ray keeps its samples up to the first whose transmittance
// drops below 1e-4; the samples behind that point need no density at all, yet they are most of
// the marched samples.  So the densities are evaluated in rounds over growing sample windows
// (below), each round only for the rays that have not stopped yet.  Each evaluated
// sample's density is the same value the full pass computes (rows are independent), so the
// kept counts, and everything after them, are unchanged.
// ---------------------------------------------------------------------------------------------
// Two rounds: round 0 evaluates the first `first_window` samples of every ray (by default
// kFirstWindow), round 1 all remaining samples of the rays still going.  A caller whose rays
// rarely stop inside the first window (the first training steps, while every density is low)
// passes first_window = all, and the evaluation takes one round.
constexpr uint32_t kFirstWindow = 48u;
constexpr uint32_t kAllSamples  = 0xFFFFFFFFu;
constexpr uint32_t kListThreads = 256u;
constexpr uint32_t kMlpWeights  = 10240u;  // packed MLP weights before the grid in the parameter vector

struct ProgressParams {
    uint32_t rays_per_batch;
    const uint32_t* ray_counter;
    const uint32_t* numsteps;   // [ray][2] (steps, base)
    const __half* density;      // raw density of sample j at density[j * density_stride] (evaluated samples only)
    uint32_t density_stride;    // 1 (density array) or 16 (network output rows, density in channel 3)
    const float* coords;
    uint32_t* kept;             // [ray]
    uint32_t* steps;            // [ray]
    float* T;                   // [ray] transmittance after the evaluated samples
    uint32_t* active;           // [ray] 1 while the ray needs more samples
    uint32_t* list_off;         // [ray] offset of the ray's rows in its list block
    uint32_t* list_totals;      // [ray blocks of kListThreads]
    uint32_t* rows;             // row list (sample indices)
    uint32_t* n_rows;           // device count of the row list
    uint32_t* block_totals;     // [ray blocks of kRaysPerCta] kept totals for the compaction
    uint32_t first_window;      // samples per ray in round 0
    uint32_t n_rounds;          // 1 (first_window covers every sample) or 2
    uint32_t* still_active;     // optional: += the rays still going after round 0
};

__device__ __forceinline__ uint32_t progress_rays(const ProgressParams& p) {
    return min(p.ray_counter != nullptr ? *p.ray_counter : p.rays_per_batch, p.rays_per_batch);
}

// Samples [lo, hi) of ray i evaluated in round `round` (empty once the ray has stopped).
__device__ __forceinline__ void round_range(const ProgressParams& p, uint32_t round, uint32_t i, uint32_t& lo, uint32_t& hi) {
    const uint32_t steps = p.numsteps[2u * i];
    lo                   = round == 0 ? 0u : min(p.first_window, steps);
    hi                   = round == 0 ? min(p.first_window, steps) : (p.active[i] ? steps : lo);
}

// Per ray: its row count in this round, exclusive offsets within blocks of kListThreads rays.
__global__ void __launch_bounds__(kListThreads) list_count_kernel(const __grid_constant__ ProgressParams p, uint32_t round) {
    const uint32_t n = progress_rays(p);
    const uint32_t i = blockIdx.x * kListThreads + threadIdx.x;
    uint32_t cnt     = 0;
    if (i < n) {
        uint32_t lo, hi;
        round_range(p, round, i, lo, hi);
        cnt = hi - lo;
    }
    uint32_t total;
    const uint32_t off = block_exclusive_scan(cnt, total);
    if (i < n) p.list_off[i] = off;
    if (threadIdx.x == 0) p.list_totals[blockIdx.x] = total;
}

// Row list of this round: the sample indices of every ray's range, in ray order.
__global__ void __launch_bounds__(kCtaThreads) list_write_kernel(const __grid_constant__ ProgressParams p, uint32_t round) {
    const uint32_t n    = progress_rays(p);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t i    = blockIdx.x * kRaysPerCta + warp;
    if (i >= n) return;
    uint32_t lo, hi;
    round_range(p, round, i, lo, hi);
    const uint32_t dst  = p.list_totals[i / kListThreads] + p.list_off[i];
    const uint32_t base = p.numsteps[2u * i + 1u];
    for (uint32_t j = lane; j < hi - lo; j += 32u) p.rows[dst + j] = base + lo + j;
}

// Transmittance over this round's samples (pass 1's loop, resumed where the last round ended).
// The last round also writes the per-CTA kept totals for the compaction.
__global__ void __launch_bounds__(kCtaThreads) keep_round_kernel(const __grid_constant__ ProgressParams p, uint32_t round) {
    __shared__ uint32_t s_kept[kRaysPerCta];
    const uint32_t n    = progress_rays(p);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t i    = blockIdx.x * kRaysPerCta + warp;
    uint32_t kept       = 0;
    if (i < n) {
        const uint32_t steps = p.numsteps[2u * i], base = p.numsteps[2u * i + 1u];
        float T              = round == 0 ? 1.0f : p.T[i];
        kept                 = round == 0 ? 0u : p.kept[i];
        const bool run       = round == 0 || p.active[i];
        bool stopped         = false;
        if (run) {
            uint32_t lo, hi;
            round_range(p, round, i, lo, hi);
            const __half* dens = p.density + static_cast<uint64_t>(base) * p.density_stride;
            const float* c     = p.coords + static_cast<uint64_t>(base) * 7u;
            // the next chunk's density and dt are loaded before this chunk is walked, so a long
            // ray pays one memory latency, not one per chunk
            auto load = [&](uint32_t j, float& d, float& dt) {
                const bool v = j < hi;
                d            = v ? __half2float(dens[static_cast<uint64_t>(j) * p.density_stride]) : 0.0f;
                dt           = v ? c[static_cast<uint64_t>(j) * 7u + 3u] : 0.0f;
            };
            // (three chunks in flight: a long ray's chunks are short to walk but far from the SM)
            float d1, dt1, d2, dt2, d3, dt3;
            load(lo + lane, d1, dt1);
            load(lo + 32u + lane, d2, dt2);
            load(lo + 64u + lane, d3, dt3);
            for (uint32_t c0 = lo; c0 < hi; c0 += 32u) {
                const uint32_t j  = c0 + lane;
                const bool valid  = j < hi;
                const float d = d1, dt = dt1;
                d1 = d2, dt1 = dt2, d2 = d3, dt2 = dt3;
                load(j + 96u, d3, dt3);
                const float alpha = valid ? 1.0f - __expf(-expf(d) * dt) : 0.0f;
                const float Tb    = prefix_transmittance(T, 1.0f - alpha, min(32u, hi - c0));
                const bool keep   = valid && !(Tb < kTransmittanceEps);
                const uint32_t nk = __popc(__ballot_sync(0xFFFFFFFFu, keep));
                if (nk > 0) T = __shfl_sync(0xFFFFFFFFu, Tb * (1.0f - alpha), nk - 1u);
                kept += nk;
                if (nk < min(32u, hi - c0)) {
                    stopped = true;
                    break;
                }
            }
            if (lane == 0) {
                p.kept[i]   = kept;
                p.T[i]      = T;
                p.active[i] = (!stopped && hi < steps) ? 1u : 0u;
                if (round == 0) p.steps[i] = steps;
            }
        }
    }
    if (round + 1u < p.n_rounds) {
        // rays still going after this round (one atomic per CTA)
        if (p.still_active != nullptr) {
            if (lane == 0) s_kept[warp] = (i < n && p.active[i]) ? 1u : 0u;
            __syncthreads();
            if (threadIdx.x == 0) {
                uint32_t a = 0;
                for (uint32_t w = 0; w < kRaysPerCta; ++w) a += s_kept[w];
                if (a) atomicAdd(p.still_active, a);
            }
        }
        return;
    }
    if (lane == 0) s_kept[warp] = kept;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t total = 0;
        for (uint32_t w = 0; w < kRaysPerCta; ++w) total += s_kept[w];
        p.block_totals[blockIdx.x] = total;
    }
}

// Selection instead of compaction: ray i's kept samples are listed as batch rows
// rows[cbase + j] = base + j (the samples stay where the march wrote them); numsteps becomes
// (kept, compacted base); *n_selected = the end of the last listed ray (the batch plus at most
// one straddling ray).
__global__ void __launch_bounds__(kCtaThreads) select_write_kernel(const __grid_constant__ KeepParams p, uint32_t* __restrict__ rows,
                                                                   uint32_t* __restrict__ sample_base, uint32_t* __restrict__ n_selected) {
    const uint32_t n    = keep_rays(p);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t i    = blockIdx.x * kRaysPerCta + warp;
    uint32_t cbase      = p.block_totals[blockIdx.x];
    for (uint32_t w = 0; w < warp; ++w) {
        const uint32_t q = blockIdx.x * kRaysPerCta + w;
        cbase += q < n ? p.kept[q] : 0u;
    }
    if (i >= n) return;
    const uint32_t k    = cbase < kNetworkBatch ? p.kept[i] : 0u;
    const uint32_t base = p.numsteps[2u * i + 1u];
    __syncwarp();
    if (lane == 0) {
        p.numsteps[2u * i]      = k;
        p.numsteps[2u * i + 1u] = cbase;
        sample_base[i]          = base;
        if (k > 0) atomicMax(n_selected, cbase + k);
    }
    for (uint32_t j = lane; j < k; j += 32u) rows[cbase + j] = base + j;
}

struct CompactedLossParams {
    uint32_t rays_per_batch;
    uint32_t step;
    const uint32_t* ray_counter;
    const uint8_t* pixels;
    uint32_t frame_count, width, height;
    const __half* output;          // [kCompactedRows][16] network output of the compacted rows
    const uint32_t* ray_indices;
    const float* rays;
    uint32_t* numsteps;            // (kept, compacted base) in; (samples in the batch, base) out
    const float* coords;           // compacted records
    __half* dloss_doutput;         // [batch][16]
    float* loss_output;
    const uint32_t* steps;         // scratch from the keep pass
    const uint32_t* sample_base;   // optional: ray i's samples are at sample_base[i] (else at its compacted base)
    int loss_kind;                 // kLossL2 (the reference) or kLossHuber
};

// Inclusive warp scans (Kogge-Stone over shfl_up): lane l gets x_0 * ... * x_l (or the sum).
__device__ __forceinline__ float warp_scan_mul(float x) {
    const uint32_t lane = threadIdx.x & 31u;
#pragma unroll
    for (uint32_t d = 1; d < 32u; d <<= 1) {
        const float y = __shfl_up_sync(0xFFFFFFFFu, x, d);
        if (lane >= d) x *= y;
    }
    return x;
}
__device__ __forceinline__ float3 warp_scan_add3(float3 v) {
    const uint32_t lane = threadIdx.x & 31u;
#pragma unroll
    for (uint32_t d = 1; d < 32u; d <<= 1) {
        const float x = __shfl_up_sync(0xFFFFFFFFu, v.x, d), y = __shfl_up_sync(0xFFFFFFFFu, v.y, d), z = __shfl_up_sync(0xFFFFFFFFu, v.z, d);
        if (lane >= d) v.x += x, v.y += y, v.z += z;
    }
    return v;
}

// One 32-sample chunk of a ray: this lane's raw network output (rgb, density) and dt, loaded a
// chunk ahead of their use; then its opacity and colour.
struct ChunkRaw {
    uint2 o;
    float dt;
};
__device__ __forceinline__ ChunkRaw chunk_load(const __half* __restrict__ out, const float* __restrict__ cin, uint32_t j, bool valid) {
    ChunkRaw raw{make_uint2(0u, 0u), 0.0f};
    if (valid) {
        raw.o  = *reinterpret_cast<const uint2*>(out + static_cast<uint64_t>(j) * 16u);
        raw.dt = cin[static_cast<uint64_t>(j) * 7u + 3u];
    }
    return raw;
}
__device__ __forceinline__ void chunk_sample(const ChunkRaw& raw, bool valid, float& alpha, float3& col, float& md, float& dt) {
    const __half2* h = reinterpret_cast<const __half2*>(&raw.o);
    const float2 rg = __half22float2(h[0]), bd = __half22float2(h[1]);
    md    = bd.y;
    dt    = raw.dt;
    alpha = valid ? 1.0f - __expf(-expf(md) * dt) : 0.0f;
    col   = {sigmoidf_(rg.x), sigmoidf_(rg.y), sigmoidf_(bd.x)};
}

// Step 5: compositing over the compacted outputs (pass 1), the loss, then the per-sample gradients
// (pass 2), for the kRaysPerCta rays of a CTA.
//
// Work split: the rays' 32-sample chunks, in ray order, form one list that is cut into
// kRaysPerCta equal contiguous ranges, one per warp, so that a long ray (hundreds of samples in
// the first steps, when the whole grid is occupied) is composited by several warps at once
// instead of one warp walking it alone.  A warp's range is a sequence of pieces, the chunks of
// one ray inside the range.  Pass 1 composites each piece from transmittance 1 (its transmittance
// product P and colour sum S); the pieces of a ray are then joined in order (transmittance and
// colour at the start of each piece; the ray's colour sum_pieces T_start * S); pass 2 recomputes
// each piece's samples from its start values.  Within a chunk the transmittance prefix and the
// colour prefix are warp scans.  (The reference walks each ray sequentially in one thread,
// ngp.train.cu:804-859; the products and sums here associate differently, a relative change of
// the order of 1e-7.)
__global__ void __launch_bounds__(kCtaThreads) loss_compacted_kernel(const __grid_constant__ CompactedLossParams p) {
    __shared__ uint32_t s_k[kRaysPerCta], s_cn[kRaysPerCta], s_src[kRaysPerCta], s_cbase[kRaysPerCta], s_first[kRaysPerCta + 1];
    __shared__ float s_P[kRaysPerCta][kRaysPerCta], s_T0[kRaysPerCta][kRaysPerCta];  // [warp][ray]
    __shared__ float3 s_S[kRaysPerCta][kRaysPerCta], s_A0[kRaysPerCta][kRaysPerCta];
    __shared__ float3 s_rgb[kRaysPerCta], s_grad[kRaysPerCta];
    const uint32_t n    = min(p.ray_counter != nullptr ? *p.ray_counter : p.rays_per_batch, p.rays_per_batch);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    if (blockIdx.x * kRaysPerCta >= n) return;  // uniform over the CTA
    if (threadIdx.x < kRaysPerCta) {
        const uint32_t i = blockIdx.x * kRaysPerCta + threadIdx.x;
        uint32_t k = 0, cn = 0, cbase = 0;
        if (i < n) {
            k     = p.numsteps[2u * i];
            cbase = p.numsteps[2u * i + 1u];
            cn    = cbase < kNetworkBatch ? min(k, kNetworkBatch - cbase) : 0u;
            p.numsteps[2u * i] = cn;
        }
        s_k[threadIdx.x]     = cn == 0 ? 0u : k;  // a ray with no sample in the batch is skipped
        s_cn[threadIdx.x]    = cn;
        s_cbase[threadIdx.x] = cbase;
        s_src[threadIdx.x]   = (i < n && p.sample_base != nullptr) ? p.sample_base[i] : cbase;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t c = 0;
        for (uint32_t r = 0; r < kRaysPerCta; ++r) {
            s_first[r] = c;
            c += (s_k[r] + 31u) / 32u;
        }
        s_first[kRaysPerCta] = c;
    }
    __syncthreads();
    const uint32_t total = s_first[kRaysPerCta];
    const uint32_t len   = (total + kRaysPerCta - 1u) / kRaysPerCta;
    const uint32_t lo = min(total, warp * len), hi = min(total, lo + len);

    // this warp's ray (for the join and the loss): its target and background, drawn while the
    // compositing runs
    const uint32_t my_i = blockIdx.x * kRaysPerCta + warp;
    float3 bg{}, target{};
    if (s_k[warp] > 0)
        ray_target(p.step, p.rays_per_batch, p.pixels, p.frame_count, p.width, p.height, p.ray_indices != nullptr ? p.ray_indices[my_i] : my_i, bg,
                   target);

    // ---- pass 1: each piece composited from transmittance 1 ----
    {
        uint32_t r = 0;
        for (uint32_t c = lo; c < hi;) {
            while (c >= s_first[r + 1u]) ++r;
            const uint32_t e = min(hi, s_first[r + 1u]);
            const __half* out = p.output + static_cast<uint64_t>(s_src[r]) * 16u;
            const float* cin  = p.coords + static_cast<uint64_t>(s_src[r]) * 7u;
            const uint32_t k  = s_k[r];
            float P   = 1.0f;
            float3 S  = {0.f, 0.f, 0.f};
            ChunkRaw next = chunk_load(out, cin, (c - s_first[r]) * 32u + lane, (c - s_first[r]) * 32u + lane < k);
            for (; c < e; ++c) {
                const uint32_t j = (c - s_first[r]) * 32u + lane;
                const ChunkRaw raw = next;
                if (c + 1u < e) next = chunk_load(out, cin, j + 32u, j + 32u < k);
                float alpha, md, dt;
                float3 col;
                chunk_sample(raw, j < k, alpha, col, md, dt);
                const float Q  = warp_scan_mul(1.0f - alpha);            // product through this sample
                const float Qu = __shfl_up_sync(0xFFFFFFFFu, Q, 1);  // every lane takes part in the shuffle
                const float Qx = lane == 0 ? 1.0f : Qu;           // product before this sample
                const float w  = alpha * (P * Qx);
                const float3 a = warp_scan_add3({w * col.x, w * col.y, w * col.z});
                S.x += __shfl_sync(0xFFFFFFFFu, a.x, 31);
                S.y += __shfl_sync(0xFFFFFFFFu, a.y, 31);
                S.z += __shfl_sync(0xFFFFFFFFu, a.z, 31);
                P *= __shfl_sync(0xFFFFFFFFu, Q, 31);
            }
            if (lane == 0) {
                s_P[warp][r] = P;
                s_S[warp][r] = S;
            }
        }
    }
    __syncthreads();

    // ---- join the pieces of this warp's ray; loss and its gradient ----
    if (s_k[warp] > 0) {
        const uint32_t r = warp;
        float T          = 1.0f;
        float3 rgb       = {0.f, 0.f, 0.f};
        for (uint32_t w = s_first[r] / len; w * len < s_first[r + 1u]; ++w) {
            if (lane == 0) {
                s_T0[w][r] = T;
                s_A0[w][r] = rgb;
            }
            const float3 S = s_S[w][r];
            rgb.x          = __fmaf_rn(T, S.x, rgb.x);
            rgb.y          = __fmaf_rn(T, S.y, rgb.y);
            rgb.z          = __fmaf_rn(T, S.z, rgb.z);
            T *= s_P[w][r];
        }
        if (s_k[r] == p.steps[my_i]) {
            rgb.x = __fmaf_rn(T, bg.x, rgb.x);
            rgb.y = __fmaf_rn(T, bg.y, rgb.y);
            rgb.z = __fmaf_rn(T, bg.z, rgb.z);
        }
        const float3 diff = {rgb.x - target.x, rgb.y - target.y, rgb.z - target.z};
        if (p.loss_output != nullptr && lane == 0) p.loss_output[my_i] = loss_value(diff, p.loss_kind, p.rays_per_batch);
        if (lane == 0) {
            s_rgb[r]  = rgb;
            s_grad[r] = loss_gradient(diff, p.loss_kind);
        }
    }
    __syncthreads();

    // ---- pass 2: per-sample gradients of the first cn samples of each ray ----
    const float scale = kLossScale / static_cast<float>(p.rays_per_batch);
    {
        uint32_t r = 0;
        for (uint32_t c = lo; c < hi;) {
            while (c >= s_first[r + 1u]) ++r;
            const uint32_t e  = min(hi, s_first[r + 1u]);
            const uint32_t cn = s_cn[r], k = s_k[r];
            const __half* out = p.output + static_cast<uint64_t>(s_src[r]) * 16u;
            const float* cin  = p.coords + static_cast<uint64_t>(s_src[r]) * 7u;
            __half* dout      = p.dloss_doutput + static_cast<uint64_t>(s_cbase[r]) * 16u;
            const float* ray  = p.rays + static_cast<uint64_t>(blockIdx.x * kRaysPerCta + r) * 6u;
            const float3 origin = {ray[0], ray[1], ray[2]};
            const float3 rgb = s_rgb[r], grad = s_grad[r];
            float T          = s_T0[warp][r];
            float3 acc       = s_A0[warp][r];
            ChunkRaw next = chunk_load(out, cin, (c - s_first[r]) * 32u + lane, (c - s_first[r]) * 32u + lane < k);
            for (; c < e; ++c) {
                const uint32_t c0 = (c - s_first[r]) * 32u;
                if (c0 >= cn) {
                    c = e;
                    break;
                }
                const uint32_t j = c0 + lane;
                const ChunkRaw raw = next;
                if (c + 1u < e) next = chunk_load(out, cin, j + 32u, j + 32u < k);
                float alpha, md, dt;
                float3 col;
                chunk_sample(raw, j < k, alpha, col, md, dt);
                const float Q      = warp_scan_mul(1.0f - alpha);
                const float Qu     = __shfl_up_sync(0xFFFFFFFFu, Q, 1);
                const float Qx     = lane == 0 ? 1.0f : Qu;
                const float Tb     = T * Qx;
                const float weight = alpha * Tb;
                float3 a           = warp_scan_add3({weight * col.x, weight * col.y, weight * col.z});
                a                  = {acc.x + a.x, acc.y + a.y, acc.z + a.z};  // colour prefix including this sample
                const float Ta     = Tb * (1.0f - alpha);
                if (j < cn) {
                    const float* cv     = cin + static_cast<uint64_t>(j) * 7u;
                    const float depth   = norm3df(cv[0] - origin.x, cv[1] - origin.y, cv[2] - origin.z);
                    const float3 suffix = {rgb.x - a.x, rgb.y - a.y, rgb.z - a.z};
                    const float g0      = scale * (weight * grad.x * (col.x * (1.0f - col.x)));
                    const float g1      = scale * (weight * grad.y * (col.y * (1.0f - col.y)));
                    const float g2      = scale * (weight * grad.z * (col.z * (1.0f - col.z)));
                    const float dd      = expf(fminf(fmaxf(md, -15.0f), 15.0f));
                    const float sum = __fmaf_rn(grad.z, __fmaf_rn(Ta, col.z, -suffix.z),
                                                __fmaf_rn(grad.x, __fmaf_rn(Ta, col.x, -suffix.x), grad.y * __fmaf_rn(Ta, col.y, -suffix.y)));
                    const float g3 = __fmaf_rn(scale, dd * (dt * sum), (md > -10.0f && depth < 0.1f) ? 1e-4f : 0.0f);
                    uint4* d       = reinterpret_cast<uint4*>(dout + static_cast<uint64_t>(j) * 16u);
                    __half2 h01 = __floats2half2_rn(g0, g1), h23 = __floats2half2_rn(g2, g3);
                    d[0]        = make_uint4(*reinterpret_cast<uint32_t*>(&h01), *reinterpret_cast<uint32_t*>(&h23), 0u, 0u);
                    d[1]        = make_uint4(0u, 0u, 0u, 0u);
                }
                T   = __shfl_sync(0xFFFFFFFFu, Ta, 31);
                acc = {__shfl_sync(0xFFFFFFFFu, a.x, 31), __shfl_sync(0xFFFFFFFFu, a.y, 31), __shfl_sync(0xFFFFFFFFu, a.z, 31)};
            }
        }
    }
}

// Padding of a selected batch: rows [n, batch) repeat rows [0, n) and their gradients scaled by
// n / batch (K12 + K13 on the row list instead of copied records).
__global__ void pad_rows_kernel(const uint32_t* __restrict__ count, uint32_t* __restrict__ rows, __half* __restrict__ dloss, uint32_t batch) {
    const uint32_t n = *count;
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (n == 0 || r < n || r >= batch) return;
    const uint32_t src = r % n;
    rows[r]            = rows[src];
    const float s      = static_cast<float>(n) / static_cast<float>(batch);
#pragma unroll
    for (int q = 0; q < 16; ++q)
        dloss[static_cast<uint64_t>(r) * 16u + q] = __float2half(__half2float(dloss[static_cast<uint64_t>(src) * 16u + q]) * s);
}

// K12 + K13 (ngp.train.cu:862-874): fill the batch tail [n, batch) by wrap-around copies of the
// first n samples; the copied gradients are scaled by n / batch.
__global__ void pad_batch_kernel(const uint32_t* __restrict__ count, float* __restrict__ coords, __half* __restrict__ dloss, uint32_t batch,
                                 __half* __restrict__ enc, uint32_t enc_stride) {
    const uint32_t n = *count;
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;  // row of the batch
    if (n == 0 || r < n || r >= batch) return;
    const uint32_t src = r % n;
    if (enc != nullptr && rows_layout(enc_stride)) {
        uint4* e = reinterpret_cast<uint4*>(enc);
#pragma unroll
        for (uint32_t q = 0; q < 4u; ++q) e[static_cast<uint64_t>(r) * 4u + q] = e[static_cast<uint64_t>(src) * 4u + q];
    } else if (enc != nullptr) {
#pragma unroll 8
        for (uint32_t f = 0; f < 32u; ++f) enc[static_cast<uint64_t>(f) * enc_stride + r] = enc[static_cast<uint64_t>(f) * enc_stride + src];
    }
#pragma unroll
    for (int q = 0; q < 7; ++q) coords[static_cast<uint64_t>(r) * 7u + q] = coords[static_cast<uint64_t>(src) * 7u + q];
    const float s = static_cast<float>(n) / static_cast<float>(batch);
#pragma unroll
    for (int q = 0; q < 16; ++q)
        dloss[static_cast<uint64_t>(r) * 16u + q] = __float2half(__half2float(dloss[static_cast<uint64_t>(src) * 16u + q]) * s);
}

// Final colour of one evaluation pixel (K10's epilogue, ngp.train.cu:715-745): clamp to [0,1],
// squared error against the sRGB target (returned), optional side-by-side comparison pixels
// (target left, render right) and rendered colour.
__device__ __forceinline__ double eval_pixel_out(uint32_t gp, float3 rgb, uint32_t image, uint32_t width, uint32_t height,
                                                 const uint8_t* __restrict__ pixels, uint8_t* __restrict__ comparison,
                                                 float* __restrict__ rendered) {
    const uint32_t px = gp % width, py = gp / width;
    double se         = 0.0;
    const float3 pr   = {fminf(fmaxf(rgb.x, 0.0f), 1.0f), fminf(fmaxf(rgb.y, 0.0f), 1.0f), fminf(fmaxf(rgb.z, 0.0f), 1.0f)};
    if (pixels != nullptr) {
        const float4 tx = read_texel(px, py, image, width, height, pixels);
        const float3 tg = {fminf(fmaxf(linear_to_srgb_c(tx.x), 0.0f), 1.0f), fminf(fmaxf(linear_to_srgb_c(tx.y), 0.0f), 1.0f),
                           fminf(fmaxf(linear_to_srgb_c(tx.z), 0.0f), 1.0f)};
        const double dr = static_cast<double>(pr.x) - tg.x, dg = static_cast<double>(pr.y) - tg.y, db = static_cast<double>(pr.z) - tg.z;
        se              = dr * dr + dg * dg + db * db;
        if (comparison != nullptr) {
            const uint64_t row = static_cast<uint64_t>(py) * width * 6u;
            uint8_t* t         = comparison + row + px * 3u;
            uint8_t* q         = comparison + row + (static_cast<uint64_t>(width) + px) * 3u;
            t[0] = static_cast<uint8_t>(tg.x * 255.0f + 0.5f), t[1] = static_cast<uint8_t>(tg.y * 255.0f + 0.5f),
            t[2] = static_cast<uint8_t>(tg.z * 255.0f + 0.5f);
            q[0] = static_cast<uint8_t>(pr.x * 255.0f + 0.5f), q[1] = static_cast<uint8_t>(pr.y * 255.0f + 0.5f),
            q[2] = static_cast<uint8_t>(pr.z * 255.0f + 0.5f);
        }
    }
    if (rendered != nullptr) {
        float* o = rendered + static_cast<uint64_t>(gp) * 3u;
        o[0] = pr.x, o[1] = pr.y, o[2] = pr.z;
    }
    return se;
}

// Front-to-back compositing of samples [base, base + steps) onto (T, rgb), stopping once the
// transmittance falls below 1e-4 (K10's loop, ngp.train.cu:690-713).  Returns true if it stopped.
__device__ __forceinline__ bool composite_samples(uint32_t base, uint32_t steps, const float* __restrict__ coords,
                                                  const __half* __restrict__ network_output, float& T, float3& rgb) {
    for (uint32_t j = 0; j < steps; ++j) {
        float r, g, b, d;
        load_output(network_output + (static_cast<uint64_t>(base) + j) * 16u, r, g, b, d);
        const float alpha  = 1.0f - __expf(-expf(d) * coords[(static_cast<uint64_t>(base) + j) * 7u + 3u]);
        const float weight = alpha * T;
        rgb.x              = __fmaf_rn(weight, sigmoidf_(r), rgb.x);
        rgb.y              = __fmaf_rn(weight, sigmoidf_(g), rgb.y);
        rgb.z              = __fmaf_rn(weight, sigmoidf_(b), rgb.z);
        T *= 1.0f - alpha;
        if (T < kTransmittanceEps) return true;
    }
    return false;
}

// Block sum of the per-thread squared errors, one fp64 atomic per CTA.
__device__ __forceinline__ void add_block_sse(double se, double* __restrict__ sse) {
#pragma unroll
    for (uint32_t o = 16; o > 0; o >>= 1) se += __shfl_down_sync(0xFFFFFFFFu, se, o);
    __shared__ double ws[kThreads / 32];
    if ((threadIdx.x & 31u) == 0) ws[threadIdx.x >> 5] = se;
    __syncthreads();
    if (threadIdx.x == 0 && sse != nullptr) {
        double tot = 0.0;
        for (uint32_t w = 0; w < kThreads / 32; ++w) tot += ws[w];
        atomicAdd(sse, tot);
    }
}

// Evaluation compositing (K10, ngp.train.cu:676-745) for a set of pixels of one image.
__global__ void __launch_bounds__(kThreads) eval_composite_kernel(uint32_t n_pixels, uint32_t pixel_offset, uint32_t image, uint32_t width,
                                                                  uint32_t height, const uint8_t* __restrict__ pixels,
                                                                  const uint32_t* __restrict__ numsteps, const float* __restrict__ coords,
                                                                  const __half* __restrict__ network_output, double* __restrict__ sse,
                                                                  uint8_t* __restrict__ comparison, float* __restrict__ rendered) {
    const uint32_t i = blockIdx.x * kThreads + threadIdx.x;
    double se        = 0.0;
    if (i < n_pixels) {
        float T    = 1.0f;
        float3 rgb = {0.0f, 0.0f, 0.0f};
        composite_samples(numsteps[2u * i + 1u], numsteps[2u * i], coords, network_output, T, rgb);
        se = eval_pixel_out(pixel_offset + i, rgb, image, width, height, pixels, comparison, rendered);
    }
    add_block_sse(se, sse);
}

// Segmented evaluation compositing: entry k (ray list[k]) of a segmented march continues its
// ray's compositing state (T, rgb) over the segment's samples -- the same sequence of float
// operations as one pass over all samples.  A ray whose transmittance fell below 1e-4, or whose
// march ended, writes its pixel; the others keep their state and are listed for the next
// segment, as are the entries past the segment's sample limit (not marched).
struct SegCompositeParams {
    uint32_t max_entries;
    const uint32_t* n_entries;  // device entry count (null: max_entries)
    const uint32_t* complete;   // entries [0, *complete) were marched
    const uint32_t* list;       // null: entry k is ray k (first segment)
    const uint32_t* numsteps;
    const float* coords;
    const __half* output;
    const float* t_out;
    float* t_state;
    uint32_t* marched;
    float4* state;              // [ray] (T, r, g, b)
    int first;
    uint32_t* next_list;
    uint32_t* next_count;
    uint32_t pixel_offset, image, width, height;
    const uint8_t* pixels;
    double* sse;
    uint8_t* comparison;
    float* rendered;
    PixelMap map;               // pixel of slot pixel_offset + ray (linear unless tiles)
};

// Compositing of one ray's segment by one warp, lane j on sample c0 + j: the transmittance
// prefix and the colour sum are taken in sample order (prefix_transmittance and ordered
// shuffles), so T and rgb are those of the sequential loop, bit for bit; stops after the first
// sample whose transmittance falls below 1e-4, as the loop does.  Returns true if it stopped.
__device__ __forceinline__ bool composite_samples_warp(uint32_t base, uint32_t steps, const float* __restrict__ coords,
                                                       const __half* __restrict__ network_output, float& T, float3& rgb) {
    const uint32_t lane = threadIdx.x & 31u;
    for (uint32_t c0 = 0; c0 < steps; c0 += 32u) {
        const uint32_t j   = c0 + lane;
        const uint32_t nv  = min(32u, steps - c0);
        const bool valid   = lane < nv;
        float r = 0.f, g = 0.f, b = 0.f, d = 0.f, dt = 0.f;
        if (valid) {
            load_output(network_output + (static_cast<uint64_t>(base) + j) * 16u, r, g, b, d);
            dt = coords[(static_cast<uint64_t>(base) + j) * 7u + 3u];
        }
        const float alpha   = valid ? 1.0f - __expf(-expf(d) * dt) : 0.0f;
        const float Tb      = prefix_transmittance(T, 1.0f - alpha, nv);
        const float Ta      = Tb * (1.0f - alpha);
        const float w       = alpha * Tb;
        const float3 col    = {sigmoidf_(r), sigmoidf_(g), sigmoidf_(b)};
        const uint32_t stop = __ballot_sync(0xFFFFFFFFu, valid && Ta < kTransmittanceEps);
        const uint32_t nk   = stop ? static_cast<uint32_t>(__ffs(stop)) : nv;
        for (uint32_t q = 0; q < nk; ++q) {
            const float wq = __shfl_sync(0xFFFFFFFFu, w, q);
            rgb.x          = __fmaf_rn(wq, __shfl_sync(0xFFFFFFFFu, col.x, q), rgb.x);
            rgb.y          = __fmaf_rn(wq, __shfl_sync(0xFFFFFFFFu, col.y, q), rgb.y);
            rgb.z          = __fmaf_rn(wq, __shfl_sync(0xFFFFFFFFu, col.z, q), rgb.z);
        }
        T = __shfl_sync(0xFFFFFFFFu, Ta, nk - 1u);
        if (stop) return true;
    }
    return false;
}

// One warp per entry (kThreads / 32 entries per CTA).
__global__ void __launch_bounds__(kThreads) seg_composite_kernel(const __grid_constant__ SegCompositeParams p) {
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t k    = blockIdx.x * (kThreads / 32u) + (threadIdx.x >> 5);
    const uint32_t n    = p.n_entries != nullptr ? min(*p.n_entries, p.max_entries) : p.max_entries;
    double se           = 0.0;
    if (k < n) {
        const uint32_t i = p.list != nullptr ? p.list[k] : k;
        bool carry       = true;  // entries past the segment's limit were not marched: unchanged
        if (k < *p.complete) {
            float T       = 1.0f;
            float3 rgb    = {0.0f, 0.0f, 0.0f};
            uint32_t done = 0;
            if (!p.first) {
                const float4 st = p.state[i];
                T = st.x, rgb = {st.y, st.z, st.w};
                done = p.marched[i];
            }
            const uint32_t steps = p.numsteps[2u * k];
            const bool stopped   = composite_samples_warp(p.numsteps[2u * k + 1u], steps, p.coords, p.output, T, rgb);
            const float t_next   = p.t_out[k];
            carry                = !(stopped || t_next < 0.0f);
            if (lane == 0) {
                uint32_t gp = 0;
                if (!carry) {
                    if (map_pixel(p.map, p.pixel_offset + i, p.width, p.height, gp))
                        se = eval_pixel_out(gp, rgb, p.image, p.width, p.height, p.pixels, p.comparison, p.rendered);
                } else {
                    p.state[i]   = make_float4(T, rgb.x, rgb.y, rgb.z);
                    p.t_state[i] = t_next;
                    p.marched[i] = done + steps;
                }
            }
        }
        if (carry && lane == 0) p.next_list[atomicAdd(p.next_count, 1u)] = i;
    }
    add_block_sse(se, p.sse);
}

constexpr size_t loss_scratch_size(uint32_t max_rays) {
    return static_cast<size_t>(max_rays) * 20u + ((max_rays + kRaysPerCta - 1u) / kRaysPerCta) * 4u +
           ((max_rays + kListThreads - 1u) / kListThreads) * 4u + 256u;
}

// The rounds of the progressive evaluation: after them p.kept holds each ray's kept count and
// every sample in front of a ray's stopping point has been evaluated, by the density network
// (density_out: raw density [samples]) or by the full network (full_out: [samples][16]).
int progressive_rounds(ProgressParams& p, uint32_t R, const ngp_grid_layout* layout, const uint16_t* params, const float* coords,
                       uint32_t sample_bound, uint16_t* enc, uint32_t enc_stride, uint16_t* density_out, uint16_t* full_out, cudaStream_t s) {
    const uint32_t warp_blocks = (R + kRaysPerCta - 1) / kRaysPerCta;
    const uint32_t list_blocks = (R + kListThreads - 1) / kListThreads;
    p.density        = reinterpret_cast<const __half*>(full_out != nullptr ? full_out + 3 : density_out);
    p.density_stride = full_out != nullptr ? 16u : 1u;
    p.n_rounds = p.first_window == kAllSamples ? 1u : 2u;
    for (uint32_t round = 0; round < p.n_rounds; ++round) {
        // rows of this round: at most its sample window per ray, and never more than all samples
        const uint64_t window = round == 0 ? p.first_window : static_cast<uint64_t>(kAllSamples) - p.first_window;
        const uint32_t bound  = static_cast<uint32_t>(std::min<uint64_t>(sample_bound, window * R));
        list_count_kernel<<<list_blocks, kListThreads, 0, s>>>(p, round);
        NGP_TRY(check_launch("list_count_kernel"));
        scan_kept_kernel<<<1, 1024, 0, s>>>(p.list_totals, list_blocks, p.n_rows, 0xFFFFFFFFu);
        NGP_TRY(check_launch("scan_kept_kernel"));
        list_write_kernel<<<warp_blocks, kCtaThreads, 0, s>>>(p, round);
        NGP_TRY(check_launch("list_write_kernel"));
        NGP_TRY(ngp_encode_grid_forward_rows(layout, bound, p.rows, p.n_rows, coords, 7, params + kMlpWeights, enc, enc_stride, s));
        if (full_out != nullptr)
            NGP_TRY(ngp_mlp_forward_rows(bound, p.rows, p.n_rows, params, enc, enc_stride, coords, 7, full_out, s));
        else
            NGP_TRY(ngp_density_forward_rows(bound, p.rows, p.n_rows, params, enc, enc_stride, density_out, s));
        keep_round_kernel<<<warp_blocks, kCtaThreads, 0, s>>>(p, round);
        NGP_TRY(check_launch("keep_round_kernel"));
    }
    return NGP_OK;
}

// Scratch layout of the progressive evaluation (ngp_loss_scratch_bytes(R) bytes).
void progress_scratch(ProgressParams& p, uint32_t R, void* scratch, uint32_t* rows) {
    const uint32_t warp_blocks = (R + kRaysPerCta - 1) / kRaysPerCta;
    const uint32_t list_blocks = (R + kListThreads - 1) / kListThreads;
    unsigned char* sc          = static_cast<unsigned char*>(scratch);
    p.steps        = reinterpret_cast<uint32_t*>(sc);
    p.kept         = reinterpret_cast<uint32_t*>(sc + static_cast<size_t>(R) * 4u);
    p.T            = reinterpret_cast<float*>(sc + static_cast<size_t>(R) * 8u);
    p.list_off     = reinterpret_cast<uint32_t*>(sc + static_cast<size_t>(R) * 12u);
    p.active       = reinterpret_cast<uint32_t*>(sc + static_cast<size_t>(R) * 16u);
    p.block_totals = reinterpret_cast<uint32_t*>(sc + static_cast<size_t>(R) * 20u);
    p.list_totals  = p.block_totals + warp_blocks;
    p.rows         = rows;
    p.n_rows       = p.list_totals + list_blocks;
}

}  // namespace
}  // namespace ngp

using namespace ngp;

extern "C" uint32_t ngp_loss_scratch_bytes(uint32_t max_rays) {
    clear_error();
    const size_t bytes = loss_scratch_size(max_rays);
    if (bytes > 0xFFFFFFFFull) {
        fail(NGP_ERR_INVALID, "loss scratch: " + std::to_string(max_rays) + " rays need " + std::to_string(bytes) +
                                  " bytes, more than a uint32 can state");
        return 0;
    }
    return static_cast<uint32_t>(bytes);
}

extern "C" int ngp_training_loss_and_compact(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels,
                                             uint32_t frame_count, uint32_t width, uint32_t height, const uint16_t* network_output,
                                             uint32_t* compacted_counter, const uint32_t* ray_indices, const float* rays, uint32_t* numsteps,
                                             const float* coords, float* compacted_coords, uint16_t* dloss_doutput, float* loss_values,
                                             void* scratch, size_t scratch_bytes, void* stream) {
    clear_error();
    if (rays_per_batch == 0) return NGP_OK;
    if (pixels == nullptr || network_output == nullptr || compacted_counter == nullptr || rays == nullptr || numsteps == nullptr ||
        coords == nullptr || compacted_coords == nullptr || dloss_doutput == nullptr || scratch == nullptr || frame_count == 0 || width == 0 ||
        height == 0)
        return fail(NGP_ERR_INVALID, "training loss: invalid input");
    if (scratch_bytes < loss_scratch_size(rays_per_batch)) return fail(NGP_ERR_INVALID, "training loss: scratch too small");
    if (reinterpret_cast<uintptr_t>(scratch) % 16u != 0) return fail(NGP_ERR_INVALID, "training loss: scratch must be 16-byte aligned");
    const cudaStream_t s  = as_stream(stream);
    const uint32_t blocks = (rays_per_batch + kRaysPerCta - 1) / kRaysPerCta;
    unsigned char* sc     = static_cast<unsigned char*>(scratch);
    LossParams p{};
    p.rays_per_batch = rays_per_batch;
    p.step           = step;
    p.ray_counter    = ray_counter;
    p.pixels         = pixels;
    p.frame_count    = frame_count;
    p.width          = width;
    p.height         = height;
    p.network_output = reinterpret_cast<const __half*>(network_output);
    p.ray_indices    = ray_indices;
    p.rays           = rays;
    p.numsteps       = numsteps;
    p.coords         = coords;
    p.coords_out     = compacted_coords;
    p.dloss_doutput  = reinterpret_cast<__half*>(dloss_doutput);
    p.loss_output    = loss_values;
    p.ray_rgb        = reinterpret_cast<float4*>(sc);
    p.kept           = reinterpret_cast<uint32_t*>(sc + static_cast<size_t>(rays_per_batch) * 16u);
    p.block_totals   = reinterpret_cast<uint32_t*>(sc + static_cast<size_t>(rays_per_batch) * 20u);
    p.batch          = kNetworkBatch;
    if (loss_values != nullptr) NGP_TRY(check_cuda(cudaMemsetAsync(loss_values, 0, sizeof(float) * rays_per_batch, s), "training loss: clear"));
    loss_pass1_kernel<<<blocks, kCtaThreads, 0, s>>>(p);
    NGP_TRY(check_launch("loss_pass1_kernel"));
    scan_kept_kernel<<<1, 1024, 0, s>>>(p.block_totals, blocks, compacted_counter, kNetworkBatch);
    NGP_TRY(check_launch("scan_kept_kernel"));
    loss_pass2_kernel<<<blocks, kCtaThreads, 0, s>>>(p);
    return check_launch("loss_pass2_kernel");
}

extern "C" uint32_t ngp_compacted_rows(void) { return kCompactedRows; }

extern "C" int ngp_training_compact_by_density(uint32_t rays_per_batch, const uint32_t* ray_counter, const uint16_t* density, const float* coords,
                                               const uint16_t* enc, uint32_t enc_stride, uint32_t* numsteps, float* compacted_coords,
                                               uint16_t* compacted_enc, uint32_t* compacted_counter, void* scratch, size_t scratch_bytes,
                                               void* stream) {
    clear_error();
    if (rays_per_batch == 0) return NGP_OK;
    if (density == nullptr || coords == nullptr || numsteps == nullptr || compacted_coords == nullptr || compacted_counter == nullptr ||
        scratch == nullptr || (compacted_enc != nullptr && enc == nullptr))
        return fail(NGP_ERR_INVALID, "compact by density: invalid input");
    if (scratch_bytes < loss_scratch_size(rays_per_batch)) return fail(NGP_ERR_INVALID, "compact by density: scratch too small");
    if (reinterpret_cast<uintptr_t>(scratch) % 16u != 0) return fail(NGP_ERR_INVALID, "compact by density: scratch must be 16-byte aligned");
    const cudaStream_t s  = as_stream(stream);
    const uint32_t blocks = (rays_per_batch + kRaysPerCta - 1) / kRaysPerCta;
    unsigned char* sc     = static_cast<unsigned char*>(scratch);
    KeepParams p{};
    p.rays_per_batch = rays_per_batch;
    p.ray_counter    = ray_counter;
    p.density        = reinterpret_cast<const __half*>(density);
    p.coords         = coords;
    p.enc            = reinterpret_cast<const __half*>(enc);
    p.enc_stride     = enc_stride;
    p.numsteps       = numsteps;
    p.coords_out     = compacted_coords;
    p.enc_out        = reinterpret_cast<__half*>(compacted_enc);
    p.steps          = reinterpret_cast<uint32_t*>(sc);
    p.kept           = reinterpret_cast<uint32_t*>(sc + static_cast<size_t>(rays_per_batch) * 4u);
    p.block_totals   = reinterpret_cast<uint32_t*>(sc + static_cast<size_t>(rays_per_batch) * 20u);
    keep_pass_kernel<<<blocks, kCtaThreads, 0, s>>>(p);
    NGP_TRY(check_launch("keep_pass_kernel"));
    scan_kept_kernel<<<1, 1024, 0, s>>>(p.block_totals, blocks, compacted_counter, kNetworkBatch);
    NGP_TRY(check_launch("scan_kept_kernel"));
    compact_copy_kernel<<<blocks, kCtaThreads, 0, s>>>(p);
    return check_launch("compact_copy_kernel");
}

extern "C" int ngp_training_compact_progressive(uint32_t rays_per_batch, const uint32_t* ray_counter, const ngp_grid_layout* layout,
                                                const uint16_t* params, const float* coords, uint32_t sample_bound, uint32_t* numsteps,
                                                uint16_t* enc, uint32_t enc_stride, uint16_t* density, uint32_t* rows, float* compacted_coords,
                                                uint16_t* compacted_enc, uint32_t* compacted_counter, void* scratch, size_t scratch_bytes,
                                                void* stream) {
    clear_error();
    if (rays_per_batch == 0) return NGP_OK;
    if (layout == nullptr || params == nullptr || coords == nullptr || numsteps == nullptr || enc == nullptr || density == nullptr || rows == nullptr ||
        compacted_coords == nullptr || compacted_counter == nullptr || scratch == nullptr || (!rows_layout(enc_stride) && enc_stride < sample_bound))
        return fail(NGP_ERR_INVALID, "progressive compaction: invalid input");
    if (scratch_bytes < loss_scratch_size(rays_per_batch)) return fail(NGP_ERR_INVALID, "progressive compaction: scratch too small");
    if (reinterpret_cast<uintptr_t>(scratch) % 16u != 0) return fail(NGP_ERR_INVALID, "progressive compaction: scratch must be 16-byte aligned");
    const cudaStream_t s       = as_stream(stream);
    const uint32_t R           = rays_per_batch;
    const uint32_t warp_blocks = (R + kRaysPerCta - 1) / kRaysPerCta;
    ProgressParams p{};
    p.first_window = kFirstWindow;
    p.rays_per_batch = R;
    p.ray_counter    = ray_counter;
    p.numsteps       = numsteps;
    p.coords         = coords;
    progress_scratch(p, R, scratch, rows);
    NGP_TRY(progressive_rounds(p, R, layout, params, coords, sample_bound, enc, enc_stride, density, nullptr, s));
    // compaction of the kept samples (as ngp_training_compact_by_density after its keep pass)
    KeepParams k{};
    k.rays_per_batch = R;
    k.ray_counter    = ray_counter;
    k.coords         = coords;
    k.enc            = reinterpret_cast<const __half*>(enc);
    k.enc_stride     = enc_stride;
    k.numsteps       = numsteps;
    k.coords_out     = compacted_coords;
    k.enc_out        = reinterpret_cast<__half*>(compacted_enc);
    k.steps          = p.steps;
    k.kept           = p.kept;
    k.block_totals   = p.block_totals;
    scan_kept_kernel<<<1, 1024, 0, s>>>(k.block_totals, warp_blocks, compacted_counter, kNetworkBatch);
    NGP_TRY(check_launch("scan_kept_kernel"));
    compact_copy_kernel<<<warp_blocks, kCtaThreads, 0, s>>>(k);
    return check_launch("compact_copy_kernel");
}

extern "C" int ngp_training_select_progressive(uint32_t rays_per_batch, const uint32_t* ray_counter, const ngp_grid_layout* layout,
                                               const uint16_t* params, const float* coords, uint32_t sample_bound, uint32_t* numsteps,
                                               uint16_t* enc, uint32_t enc_stride, uint16_t* density, uint32_t* rows, uint32_t* batch_rows,
                                               uint32_t* n_selected, uint32_t* compacted_counter, void* scratch, size_t scratch_bytes, void* stream) {
    return ngp_training_select_progressive_window(rays_per_batch, ray_counter, layout, params, coords, sample_bound, numsteps, enc, enc_stride, density,
                                                  rows, batch_rows, n_selected, compacted_counter, scratch, scratch_bytes, kFirstWindow, nullptr, stream);
}

extern "C" int ngp_training_select_progressive_window(uint32_t rays_per_batch, const uint32_t* ray_counter, const ngp_grid_layout* layout,
                                                      const uint16_t* params, const float* coords, uint32_t sample_bound, uint32_t* numsteps,
                                                      uint16_t* enc, uint32_t enc_stride, uint16_t* density, uint32_t* rows, uint32_t* batch_rows,
                                                      uint32_t* n_selected, uint32_t* compacted_counter, void* scratch, size_t scratch_bytes,
                                                      uint32_t first_window, uint32_t* still_active, void* stream) {
    clear_error();
    if (first_window == 0) return fail(NGP_ERR_INVALID, "progressive selection: the first window must hold at least one sample");
    if (rays_per_batch == 0) return NGP_OK;
    if (layout == nullptr || params == nullptr || coords == nullptr || numsteps == nullptr || enc == nullptr || density == nullptr || rows == nullptr ||
        batch_rows == nullptr || n_selected == nullptr || compacted_counter == nullptr || scratch == nullptr || (!rows_layout(enc_stride) && enc_stride < sample_bound))
        return fail(NGP_ERR_INVALID, "progressive selection: invalid input");
    if (scratch_bytes < loss_scratch_size(rays_per_batch)) return fail(NGP_ERR_INVALID, "progressive selection: scratch too small");
    if (reinterpret_cast<uintptr_t>(scratch) % 16u != 0) return fail(NGP_ERR_INVALID, "progressive selection: scratch must be 16-byte aligned");
    const cudaStream_t s       = as_stream(stream);
    const uint32_t R           = rays_per_batch;
    const uint32_t warp_blocks = (R + kRaysPerCta - 1) / kRaysPerCta;
    ProgressParams p{};
    p.first_window = kFirstWindow;
    p.rays_per_batch = R;
    p.ray_counter    = ray_counter;
    p.numsteps       = numsteps;
    p.coords         = coords;
    progress_scratch(p, R, scratch, rows);
    p.first_window = first_window;
    p.still_active = first_window == kAllSamples ? nullptr : still_active;
    if (still_active != nullptr) NGP_TRY(check_cuda(cudaMemsetAsync(still_active, 0, sizeof(uint32_t), s), "progressive selection: clear active count"));
    NGP_TRY(progressive_rounds(p, R, layout, params, coords, sample_bound, enc, enc_stride, density, nullptr, s));
    KeepParams k{};
    k.rays_per_batch = R;
    k.ray_counter    = ray_counter;
    k.numsteps       = numsteps;
    k.steps          = p.steps;
    k.kept           = p.kept;
    k.block_totals   = p.block_totals;
    scan_kept_kernel<<<1, 1024, 0, s>>>(k.block_totals, warp_blocks, compacted_counter, kNetworkBatch);
    NGP_TRY(check_launch("scan_kept_kernel"));
    NGP_TRY(check_cuda(cudaMemsetAsync(n_selected, 0, sizeof(uint32_t), s), "progressive selection: clear count"));
    select_write_kernel<<<warp_blocks, kCtaThreads, 0, s>>>(k, batch_rows, p.list_off, n_selected);
    return check_launch("select_write_kernel");
}

extern "C" int ngp_training_loss_selected_kind(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels,
                                               uint32_t frame_count, uint32_t width, uint32_t height, const uint16_t* network_output,
                                               const uint32_t* ray_indices, const float* rays, uint32_t* numsteps, const float* coords,
                                               uint16_t* dloss_doutput, float* loss_values, const void* scratch, size_t scratch_bytes, int loss_kind,
                                               void* stream) {
    clear_error();
    if (loss_kind != kLossL2 && loss_kind != kLossHuber) return fail(NGP_ERR_INVALID, "selected loss: unknown loss kind");
    if (rays_per_batch == 0) return NGP_OK;
    if (pixels == nullptr || network_output == nullptr || rays == nullptr || numsteps == nullptr || coords == nullptr || dloss_doutput == nullptr ||
        scratch == nullptr || frame_count == 0 || width == 0 || height == 0)
        return fail(NGP_ERR_INVALID, "selected loss: invalid input");
    if (scratch_bytes < loss_scratch_size(rays_per_batch)) return fail(NGP_ERR_INVALID, "selected loss: scratch too small");
    const cudaStream_t s = as_stream(stream);
    CompactedLossParams p{};
    p.rays_per_batch = rays_per_batch;
    p.step           = step;
    p.ray_counter    = ray_counter;
    p.pixels         = pixels;
    p.frame_count    = frame_count;
    p.width          = width;
    p.height         = height;
    p.output         = reinterpret_cast<const __half*>(network_output);
    p.ray_indices    = ray_indices;
    p.rays           = rays;
    p.numsteps       = numsteps;
    p.coords         = coords;
    p.dloss_doutput  = reinterpret_cast<__half*>(dloss_doutput);
    p.loss_output    = loss_values;
    p.steps          = static_cast<const uint32_t*>(scratch);
    p.sample_base    = static_cast<const uint32_t*>(scratch) + static_cast<size_t>(rays_per_batch) * 3u;  // list_off region
    p.loss_kind      = loss_kind;
    if (loss_values != nullptr) NGP_TRY(check_cuda(cudaMemsetAsync(loss_values, 0, sizeof(float) * rays_per_batch, s), "selected loss: clear"));
    loss_compacted_kernel<<<(rays_per_batch + kRaysPerCta - 1) / kRaysPerCta, kCtaThreads, 0, s>>>(p);
    return check_launch("loss_compacted_kernel");
}

extern "C" int ngp_training_loss_selected(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels,
                                          uint32_t frame_count, uint32_t width, uint32_t height, const uint16_t* network_output,
                                          const uint32_t* ray_indices, const float* rays, uint32_t* numsteps, const float* coords,
                                          uint16_t* dloss_doutput, float* loss_values, const void* scratch, size_t scratch_bytes, void* stream) {
    return ngp_training_loss_selected_kind(rays_per_batch, step, ray_counter, pixels, frame_count, width, height, network_output, ray_indices, rays,
                                           numsteps, coords, dloss_doutput, loss_values, scratch, scratch_bytes, kLossL2, stream);
}

extern "C" int ngp_pad_training_rows(const uint32_t* compacted_counter, uint32_t* batch_rows, uint16_t* dloss_doutput, void* stream) {
    clear_error();
    if (compacted_counter == nullptr || batch_rows == nullptr || dloss_doutput == nullptr) return fail(NGP_ERR_INVALID, "pad rows: null pointer");
    pad_rows_kernel<<<kNetworkBatch / 256u, 256, 0, as_stream(stream)>>>(compacted_counter, batch_rows, reinterpret_cast<__half*>(dloss_doutput),
                                                                           kNetworkBatch);
    return check_launch("pad_rows_kernel");
}

extern "C" int ngp_eval_network_progressive(uint32_t n_rays, const ngp_grid_layout* layout, const uint16_t* params, const float* coords,
                                            uint32_t sample_bound, const uint32_t* numsteps, uint16_t* enc, uint32_t enc_stride, uint16_t* network_output,
                                            uint32_t* rows, void* scratch, size_t scratch_bytes, void* stream) {
    clear_error();
    if (n_rays == 0) return NGP_OK;
    if (layout == nullptr || params == nullptr || coords == nullptr || numsteps == nullptr || enc == nullptr || network_output == nullptr ||
        rows == nullptr || scratch == nullptr || (!rows_layout(enc_stride) && enc_stride < sample_bound))
        return fail(NGP_ERR_INVALID, "progressive evaluation: invalid input");
    if (scratch_bytes < loss_scratch_size(n_rays)) return fail(NGP_ERR_INVALID, "progressive evaluation: scratch too small");
    if (reinterpret_cast<uintptr_t>(scratch) % 16u != 0) return fail(NGP_ERR_INVALID, "progressive evaluation: scratch must be 16-byte aligned");
    ProgressParams p{};
    p.first_window = kFirstWindow;
    p.rays_per_batch = n_rays;
    p.numsteps       = numsteps;
    p.coords         = coords;
    progress_scratch(p, n_rays, scratch, rows);
    return progressive_rounds(p, n_rays, layout, params, coords, sample_bound, enc, enc_stride, nullptr, network_output, as_stream(stream));
}

extern "C" int ngp_training_loss_compacted(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels,
                                           uint32_t frame_count, uint32_t width, uint32_t height, const uint16_t* compacted_output,
                                           const uint32_t* ray_indices, const float* rays, uint32_t* numsteps, const float* compacted_coords,
                                           uint16_t* dloss_doutput, float* loss_values, const void* scratch, size_t scratch_bytes, void* stream) {
    clear_error();
    if (rays_per_batch == 0) return NGP_OK;
    if (pixels == nullptr || compacted_output == nullptr || rays == nullptr || numsteps == nullptr || compacted_coords == nullptr ||
        dloss_doutput == nullptr || scratch == nullptr || frame_count == 0 || width == 0 || height == 0)
        return fail(NGP_ERR_INVALID, "compacted loss: invalid input");
    if (scratch_bytes < loss_scratch_size(rays_per_batch)) return fail(NGP_ERR_INVALID, "compacted loss: scratch too small");
    const cudaStream_t s = as_stream(stream);
    CompactedLossParams p{};
    p.rays_per_batch = rays_per_batch;
    p.step           = step;
    p.ray_counter    = ray_counter;
    p.pixels         = pixels;
    p.frame_count    = frame_count;
    p.width          = width;
    p.height         = height;
    p.output         = reinterpret_cast<const __half*>(compacted_output);
    p.ray_indices    = ray_indices;
    p.rays           = rays;
    p.numsteps       = numsteps;
    p.coords         = compacted_coords;
    p.dloss_doutput  = reinterpret_cast<__half*>(dloss_doutput);
    p.loss_output    = loss_values;
    p.steps          = static_cast<const uint32_t*>(scratch);
    if (loss_values != nullptr) NGP_TRY(check_cuda(cudaMemsetAsync(loss_values, 0, sizeof(float) * rays_per_batch, s), "compacted loss: clear"));
    loss_compacted_kernel<<<(rays_per_batch + kRaysPerCta - 1) / kRaysPerCta, kCtaThreads, 0, s>>>(p);
    return check_launch("loss_compacted_kernel");
}

extern "C" int ngp_pad_training_batch(const uint32_t* compacted_counter, float* compacted_coords, uint16_t* dloss_doutput, void* stream) {
    clear_error();
    if (compacted_counter == nullptr || compacted_coords == nullptr || dloss_doutput == nullptr) return fail(NGP_ERR_INVALID, "pad batch: null pointer");
    pad_batch_kernel<<<kNetworkBatch / 256u, 256, 0, as_stream(stream)>>>(compacted_counter, compacted_coords, reinterpret_cast<__half*>(dloss_doutput),
                                                                            kNetworkBatch, nullptr, 0u);
    return check_launch("pad_batch_kernel");
}

extern "C" int ngp_pad_training_batch_enc(const uint32_t* compacted_counter, float* compacted_coords, uint16_t* dloss_doutput, uint16_t* enc,
                                          uint32_t enc_stride, void* stream) {
    clear_error();
    if (compacted_counter == nullptr || compacted_coords == nullptr || dloss_doutput == nullptr || enc == nullptr || (!rows_layout(enc_stride) && enc_stride < kNetworkBatch))
        return fail(NGP_ERR_INVALID, "pad batch: invalid input");
    pad_batch_kernel<<<kNetworkBatch / 256u, 256, 0, as_stream(stream)>>>(compacted_counter, compacted_coords, reinterpret_cast<__half*>(dloss_doutput),
                                                                            kNetworkBatch, reinterpret_cast<__half*>(enc), enc_stride);
    return check_launch("pad_batch_kernel");
}

extern "C" int ngp_eval_composite_segment_tiles(uint32_t max_entries, const uint32_t* n_entries, const uint32_t* complete, const uint32_t* list,
                                                const uint32_t* numsteps, const float* coords, const uint16_t* network_output, const float* t_out,
                                                float* t_state, uint32_t* marched, float* state, uint32_t* next_list, uint32_t* next_count,
                                                uint32_t pixel_offset, uint32_t image, uint32_t width, uint32_t height, const uint8_t* pixels,
                                                double* sse, uint8_t* comparison, float* rendered, uint32_t first_tile, uint32_t tile_stride,
                                                void* stream) {
    clear_error();
    if (tile_stride == 0) return fail(NGP_ERR_INVALID, "segment composite: tile stride 0");
    if (max_entries == 0) return NGP_OK;
    if (complete == nullptr || numsteps == nullptr || coords == nullptr || network_output == nullptr || t_out == nullptr || t_state == nullptr ||
        marched == nullptr || state == nullptr || next_list == nullptr || next_count == nullptr || width == 0 || height == 0)
        return fail(NGP_ERR_INVALID, "segment composite: invalid input");
    if (reinterpret_cast<uintptr_t>(state) % 16u != 0) return fail(NGP_ERR_INVALID, "segment composite: state must be 16-byte aligned");
    SegCompositeParams p{};
    p.max_entries  = max_entries;
    p.n_entries    = n_entries;
    p.complete     = complete;
    p.list         = list;
    p.numsteps     = numsteps;
    p.coords       = coords;
    p.output       = reinterpret_cast<const __half*>(network_output);
    p.t_out        = t_out;
    p.t_state      = t_state;
    p.marched      = marched;
    p.state        = reinterpret_cast<float4*>(state);
    p.first        = list == nullptr ? 1 : 0;
    p.next_list    = next_list;
    p.next_count   = next_count;
    p.pixel_offset = pixel_offset;
    p.image        = image;
    p.width        = width;
    p.height       = height;
    p.pixels       = pixels;
    p.sse          = sse;
    p.comparison   = comparison;
    p.rendered     = rendered;
    p.map          = first_tile == 0xFFFFFFFFu ? PixelMap{0u, 0u, 0u} : PixelMap{(width + kTileSide - 1u) / kTileSide, first_tile, tile_stride};
    constexpr uint32_t per_cta = kThreads / 32u;
    seg_composite_kernel<<<(max_entries + per_cta - 1) / per_cta, kThreads, 0, as_stream(stream)>>>(p);
    return check_launch("seg_composite_kernel");
}

extern "C" int ngp_eval_composite_segment(uint32_t max_entries, const uint32_t* n_entries, const uint32_t* complete, const uint32_t* list,
                                          const uint32_t* numsteps, const float* coords, const uint16_t* network_output, const float* t_out,
                                          float* t_state, uint32_t* marched, float* state, uint32_t* next_list, uint32_t* next_count,
                                          uint32_t pixel_offset, uint32_t image, uint32_t width, uint32_t height, const uint8_t* pixels, double* sse,
                                          uint8_t* comparison, float* rendered, void* stream) {
    return ngp_eval_composite_segment_tiles(max_entries, n_entries, complete, list, numsteps, coords, network_output, t_out, t_state, marched, state,
                                            next_list, next_count, pixel_offset, image, width, height, pixels, sse, comparison, rendered, 0xFFFFFFFFu,
                                            1u, stream);
}

extern "C" int ngp_eval_composite(uint32_t n_pixels, uint32_t pixel_offset, uint32_t image, uint32_t width, uint32_t height, const uint8_t* pixels,
                                  const uint32_t* numsteps, const float* coords, const uint16_t* network_output, double* sse,
                                  uint8_t* comparison, float* rendered, void* stream) {
    clear_error();
    if (n_pixels == 0) return NGP_OK;
    if (numsteps == nullptr || coords == nullptr || network_output == nullptr) return fail(NGP_ERR_INVALID, "eval composite: null pointer");
    eval_composite_kernel<<<(n_pixels + kThreads - 1) / kThreads, kThreads, 0, as_stream(stream)>>>(
        n_pixels, pixel_offset, image, width, height, pixels, numsteps, coords, reinterpret_cast<const __half*>(network_output), sse, comparison,
        rendered);
    return check_launch("eval_composite_kernel");
}

// ---------------------------------------------------------------------------------------------
// Variant without any allocation.
//
// Some callers cannot allocate device memory at the point where they run the loss: code that
// runs inside a host callback or a driver-managed region where cudaMalloc is not allowed,
// runtimes that hand a plugin only fixed buffers and forbid it from growing its footprint, and
// integrations whose memory budget is fixed at start-up.  For them this entry point takes its
// scratch from one statically sized device array that every GPU loading the library holds until
// the process exits (kNoAllocScratchBytes, about 5 MiB: room for 2^18 rays).
// ---------------------------------------------------------------------------------------------
namespace {

constexpr uint32_t kNoAllocMaxRays    = 1u << 18;
constexpr size_t kNoAllocScratchBytes = loss_scratch_size(kNoAllocMaxRays);
static __device__ __align__(256) unsigned char g_noalloc_loss_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices]             = {};
unsigned long long g_noalloc_ctx[kMaxDevices] = {};

// Identity of the context current on this thread (cuCtxGetId through the runtime's driver entry
// point, so that the library needs no link against libcuda).  A device reset, or the release and
// re-creation of the primary context, gives a new identity; the module and its static array are
// then loaded again, possibly at another address.
int current_context_id(unsigned long long* id) {
    using GetCurrent = int (*)(void**);
    using GetId      = int (*)(void*, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id           = nullptr;
    if (get_current == nullptr || get_id == nullptr) {
        void* a                            = nullptr;
        void* b                            = nullptr;
        cudaDriverEntryPointQueryResult qa = cudaDriverEntryPointSymbolNotFound, qb = cudaDriverEntryPointSymbolNotFound;
        NGP_TRY(check_cuda(cudaGetDriverEntryPoint("cuCtxGetCurrent", &a, cudaEnableDefault, &qa), "no-alloc loss: cuCtxGetCurrent entry point"));
        NGP_TRY(check_cuda(cudaGetDriverEntryPoint("cuCtxGetId", &b, cudaEnableDefault, &qb), "no-alloc loss: cuCtxGetId entry point"));
        if (a == nullptr || b == nullptr || qa != cudaDriverEntryPointSuccess || qb != cudaDriverEntryPointSuccess)
            return fail(NGP_ERR_CUDA, "no-alloc loss: the driver exports no cuCtxGetCurrent / cuCtxGetId");
        get_current = reinterpret_cast<GetCurrent>(a);
        get_id      = reinterpret_cast<GetId>(b);
    }
    void* ctx = nullptr;
    if (get_current(&ctx) != 0 || ctx == nullptr) return fail(NGP_ERR_CUDA, "no-alloc loss: no current context");
    if (get_id(ctx, id) != 0) return fail(NGP_ERR_CUDA, "no-alloc loss: cuCtxGetId failed");
    return NGP_OK;
}

// Device address of this GPU's copy of the array, looked up with that device current: once per
// device and context (again after a device reset).  The host-side name of the array is not a
// device address and must never be passed to a kernel.
int noalloc_scratch(void** out) {
    int device = 0;
    NGP_TRY(check_cuda(cudaGetDevice(&device), "no-alloc loss: cudaGetDevice"));
    if (device < 0 || device >= kMaxDevices) return fail(NGP_ERR_INVALID, "no-alloc loss: device index out of range");
    // cudaSetDevice makes the device's primary context current on this thread (creating it if
    // needed), so that its identity can be read
    NGP_TRY(check_cuda(cudaSetDevice(device), "no-alloc loss: cudaSetDevice"));
    unsigned long long ctx = 0;
    NGP_TRY(current_context_id(&ctx));
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[device] == nullptr || g_noalloc_ctx[device] != ctx) {
        void* p = nullptr;
        NGP_TRY(check_cuda(cudaGetSymbolAddress(&p, g_noalloc_loss_scratch), "no-alloc loss: cudaGetSymbolAddress"));
        g_noalloc_ptr[device] = p;
        g_noalloc_ctx[device] = ctx;
    }
    *out = g_noalloc_ptr[device];
    return NGP_OK;
}

}  // namespace

extern "C" uint32_t ngp_training_loss_and_compact_noalloc_max_rays(void) { return kNoAllocMaxRays; }

extern "C" int ngp_training_loss_and_compact_noalloc(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels,
                                                     uint32_t frame_count, uint32_t width, uint32_t height, const uint16_t* network_output,
                                                     uint32_t* compacted_counter, const uint32_t* ray_indices, const float* rays,
                                                     uint32_t* numsteps, const float* coords, float* compacted_coords, uint16_t* dloss_doutput,
                                                     float* loss_values, void* stream) {
    clear_error();
    if (rays_per_batch > kNoAllocMaxRays)
        return fail(NGP_ERR_INVALID, "training loss (no-alloc): rays_per_batch " + std::to_string(rays_per_batch) + " exceeds the static scratch limit of " +
                                         std::to_string(kNoAllocMaxRays) + " rays");
    if (rays_per_batch == 0) return NGP_OK;
    void* scratch = nullptr;
    NGP_TRY(noalloc_scratch(&scratch));
    return ngp_training_loss_and_compact(rays_per_batch, step, ray_counter, pixels, frame_count, width, height, network_output, compacted_counter,
                                         ray_indices, rays, numsteps, coords, compacted_coords, dloss_doutput, loss_values, scratch,
                                         kNoAllocScratchBytes, stream);
}
