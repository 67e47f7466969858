// Occupancy density grid (update + bitfield) and ray marching with deterministic compaction.
//
// Replaces the reference's K1-K8 (ngp.train.cu:310-667) and the host wrappers
// update_density_grid / sample_training_batch / run_evaluation's sampling (1526-1595,
// 1919-1930, 1618-1642).
//
// B200 design notes:
// * Ray marching is count -> scan -> write: the count pass stores each ray's step count and a
//   per-CTA total, one CTA scans the totals, and the write pass places every ray's samples at
//   its prefix offset.  Sample order is therefore the ray order (deterministic, and coalesced
//   for the network that consumes it) instead of the reference's atomic slot order.
// * The grid mean is a fixed-order two-level reduction (deterministic), fused with the EMA.
// * The occupancy bitfield (256 KB) stays L2/L1 resident for the marching kernels.
#include <cmath>

#include "sampler.cuh"

namespace ngp {
namespace {


// ------------------------------------------------------------------------------------------
// density grid
// ------------------------------------------------------------------------------------------

// K1 (ngp.train.cu:310-381): a cell is "trained" when any corner projects into some training
// view along a ray that matches the pixel's camera ray; untrained cells get -1.
__global__ void mark_untrained_kernel(float* __restrict__ values, const CameraSet cam) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= kGridCells) return;
    const uint32_t x = morton_compact(i), y = morton_compact(i >> 1), z = morton_compact(i >> 2);
    constexpr float voxel = 1.0f / 128.0f;
    const float3 cmin     = {static_cast<float>(x) * voxel, static_cast<float>(y) * voxel, static_cast<float>(z) * voxel};
    bool trained          = false;
    for (uint32_t frame = 0; frame < cam.frame_count && !trained; ++frame) {
        const float* f  = cam.camera + static_cast<uint64_t>(frame) * 12u;
        const float3 cx = {f[0], f[1], f[2]}, cy = {f[3], f[4], f[5]}, cz = {f[6], f[7], f[8]}, o = {f[9], f[10], f[11]};
        for (uint32_t corner = 0; corner < 8 && !trained; ++corner) {
            const float3 pos = {cmin.x + ((corner & 1u) ? voxel : 0.0f), cmin.y + ((corner & 2u) ? voxel : 0.0f),
                                cmin.z + ((corner & 4u) ? voxel : 0.0f)};
            const float3 rel = {pos.x - o.x, pos.y - o.y, pos.z - o.z};
            const float dist = norm3df(rel.x, rel.y, rel.z);
            if (dist <= 0.0f) continue;
            const float lx = __fmaf_rn(rel.z, cx.z, __fmaf_rn(rel.x, cx.x, rel.y * cx.y));
            const float ly = __fmaf_rn(rel.z, cy.z, __fmaf_rn(rel.x, cy.x, rel.y * cy.y));
            const float lz = __fmaf_rn(rel.z, cz.z, __fmaf_rn(rel.x, cz.x, rel.y * cz.y));
            if (lz / dist < 1e-4f) continue;
            const float px = lx * cam.focal_x / lz + cam.principal_x;
            const float py = ly * cam.focal_y / lz + cam.principal_y;
            if (px <= 0.0f || py <= 0.0f || px >= static_cast<float>(cam.width) || py >= static_cast<float>(cam.height)) continue;
            const float rx  = (px - cam.principal_x) / cam.focal_x;
            const float ry  = (py - cam.principal_y) / cam.focal_y;
            const float3 rd = {__fmaf_rn(cx.x, rx, cy.x * ry) + cz.x, __fmaf_rn(cx.y, rx, cy.y * ry) + cz.y, __fmaf_rn(cx.z, rx, cy.z * ry) + cz.z};
            const float rl  = norm3df(rd.x, rd.y, rd.z);
            if (rl <= 0.0f) continue;
            const float3 rn = {rd.x / rl, rd.y / rl, rd.z / rl};
            const float3 dn = {rel.x / dist, rel.y / dist, rel.z / dist};
            trained         = norm3df(rn.x - dn.x, rn.y - dn.y, rn.z - dn.z) < 1e-3f;
        }
    }
    values[i] = trained ? 0.0f : -1.0f;
}

// K2 (ngp.train.cu:383-424): sample positions for the grid update.  Samples [0, n_uniform) pick
// cells uniformly; the rest take up to 10 hashed tries for a cell above the occupancy
// threshold.  Each writes a 7-float record and its cell index.
__global__ void generate_grid_samples_kernel(uint32_t n_uniform, uint32_t n_nonuniform, uint32_t ema_step, const float* __restrict__ values,
                                             float* __restrict__ coords, uint32_t* __restrict__ indices) {
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n_uniform + n_nonuniform) return;
    const bool uniform   = g < n_uniform;
    const uint32_t i     = uniform ? g : g - n_uniform;
    const uint32_t count = uniform ? n_uniform : n_nonuniform;
    const float thresh   = uniform ? -0.01f : kMinOpticalThick;
    Pcg32 rng{kTrainSeed};
    rng.advance(((static_cast<uint64_t>(ema_step) * 2ull + (uniform ? 0ull : 1ull) + 1ull) << 32u) + static_cast<uint64_t>(i) * 4ull);
    uint32_t idx = 0;
    for (uint32_t j = 0; j < 10; ++j) {
        idx = static_cast<uint32_t>(((static_cast<uint64_t>(i) + static_cast<uint64_t>(ema_step) * count) * 56924617ull +
                                     static_cast<uint64_t>(j) * 19349663ull + 96925573ull) %
                                    kGridCells);
        if (values[idx] > thresh) break;
    }
    const uint32_t x = morton_compact(idx), y = morton_compact(idx >> 1), z = morton_compact(idx >> 2);
    float* c   = coords + static_cast<uint64_t>(g) * 7u;
    c[0]       = (static_cast<float>(x) + rng.next_float()) / 128.0f;
    c[1]       = (static_cast<float>(y) + rng.next_float()) / 128.0f;
    c[2]       = (static_cast<float>(z) + rng.next_float()) / 128.0f;
    c[3]       = kConeStep;
    c[4]       = 0.5f;
    c[5]       = 0.5f;
    c[6]       = 0.5f;
    indices[g] = idx;
}

// K2 in cell order.  Sample i's first cell is ((i + ema_step * count) * 56924617 + 96925573) mod
// 2^21 (the reference's hash with j = 0): an odd multiplier makes this a bijection of [0, 2^21),
// so every cell g is the first cell of exactly one index i = (g - 96925573) * 56924617^-1 -
// ema_step * count (mod 2^21) of each sample set, and that sample exists iff i < count.  Thread g
// generates those samples (the same records and cell indices as generate_grid_samples_kernel:
// same PCG32 draws, same retries), so consecutive samples lie in consecutive Morton cells and the
// encoding of the grid samples gathers neighbouring table entries across a warp instead of
// random ones.  Only the order of the samples differs, which the update does not see: each
// sample's density is splatted with an atomic max into its own cell.
// With all 2^21 samples uniform (the first 256 steps) thread g writes slot g; otherwise a warp
// reserves its slots with one atomic on *counter (zeroed by the caller): the warp's samples stay
// in cell order, warps in any order.
__device__ __forceinline__ void grid_sample_record(uint32_t i, uint32_t count, uint32_t ema_step, float thresh, uint64_t base_state,
                                                   const uint64_t* __restrict__ jm, const uint64_t* __restrict__ jp,
                                                   const float* __restrict__ values, float* __restrict__ c, uint32_t* __restrict__ index) {
    float pos[3];
    uint32_t idx;
    grid_sample_position(i, count, ema_step, thresh, base_state, jm, jp, values, pos, idx);
    c[0]   = pos[0];
    c[1]   = pos[1];
    c[2]   = pos[2];
    c[3]   = kConeStep;
    c[4]   = 0.5f;
    c[5]   = 0.5f;
    c[6]   = 0.5f;
    *index = idx;
}

__global__ void __launch_bounds__(256) generate_grid_samples_ordered_kernel(uint32_t n_uniform, uint32_t n_nonuniform, uint32_t ema_step,
                                                                            uint64_t base_uniform, uint64_t base_nonuniform,
                                                                            const float* __restrict__ values, float* __restrict__ coords,
                                                                            uint32_t* __restrict__ indices, uint32_t* __restrict__ counter) {
    __shared__ uint64_t jm[64], jp[64];
    if (threadIdx.x < 64) jm[threadIdx.x] = c_pcg_jump.mult[threadIdx.x];
    else if (threadIdx.x < 128) jp[threadIdx.x - 64] = c_pcg_jump.plus[threadIdx.x - 64];
    __syncthreads();
    const uint32_t g   = blockIdx.x * blockDim.x + threadIdx.x;  // cell (Morton index)
    const uint32_t rel = (g - (kGridHashAdd & (kGridCells - 1u))) * kGridHashMulInv;  // i + ema_step * count (mod 2^21)
    const uint32_t iu  = (rel - ema_step * n_uniform) & (kGridCells - 1u);
    const uint32_t in  = (rel - ema_step * n_nonuniform) & (kGridCells - 1u);
    const bool has_u   = iu < n_uniform;
    const bool has_n   = in < n_nonuniform;
    uint32_t slot      = g;
    if (counter != nullptr) {
        const uint32_t lane = threadIdx.x & 31u;
        const uint32_t cnt  = static_cast<uint32_t>(has_u) + static_cast<uint32_t>(has_n);
        uint32_t incl       = cnt;
#pragma unroll
        for (uint32_t o = 1; o < 32; o <<= 1) {
            const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
            if (lane >= o) incl += v;
        }
        const uint32_t total = __shfl_sync(0xFFFFFFFFu, incl, 31);
        uint32_t base        = 0;
        if (lane == 31 && total > 0) base = atomicAdd(counter, total);
        base = __shfl_sync(0xFFFFFFFFu, base, 31);
        slot = base + incl - cnt;
    }
    if (has_u) {
        grid_sample_record(iu, n_uniform, ema_step, -0.01f, base_uniform, jm, jp, values, coords + static_cast<uint64_t>(slot) * 7u, indices + slot);
        ++slot;
    }
    if (has_n)
        grid_sample_record(in, n_nonuniform, ema_step, kMinOpticalThick, base_nonuniform, jm, jp, values, coords + static_cast<uint64_t>(slot) * 7u,
                           indices + slot);
}

// K3 (ngp.train.cu:426-432): scratch[cell] = max(scratch[cell], exp(raw density) * dt).
__global__ void splat_kernel(uint32_t n, const uint32_t* __restrict__ indices, const __half* __restrict__ density, float* __restrict__ scratch) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float thickness = expf(__half2float(density[i])) * kConeStep;
    atomicMax(reinterpret_cast<uint32_t*>(scratch + indices[i]), __float_as_uint(thickness));
}

// K4 + first level of K5 (ngp.train.cu:434-461): EMA update of every cell, then per-CTA sums of
// max(v, 0) in a fixed order.  1024 cells per CTA (256 threads x float4).
__global__ void __launch_bounds__(256) ema_partial_kernel(const float* __restrict__ scratch, float* __restrict__ values, float decay,
                                                          float* __restrict__ partial) {
    const uint32_t q = blockIdx.x * 256u + threadIdx.x;  // float4 index
    const float4 s   = reinterpret_cast<const float4*>(scratch)[q];
    float4 v         = reinterpret_cast<float4*>(values)[q];
    v.x              = v.x < 0.0f ? v.x : fmaxf(v.x * decay, s.x);
    v.y              = v.y < 0.0f ? v.y : fmaxf(v.y * decay, s.y);
    v.z              = v.z < 0.0f ? v.z : fmaxf(v.z * decay, s.z);
    v.w              = v.w < 0.0f ? v.w : fmaxf(v.w * decay, s.w);
    reinterpret_cast<float4*>(values)[q] = v;
    float sum = ((fmaxf(v.x, 0.0f) + fmaxf(v.y, 0.0f)) + fmaxf(v.z, 0.0f)) + fmaxf(v.w, 0.0f);
#pragma unroll
    for (uint32_t o = 16; o > 0; o >>= 1) sum += __shfl_down_sync(0xFFFFFFFFu, sum, o);
    __shared__ float warp_sum[8];
    if ((threadIdx.x & 31u) == 0) warp_sum[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x == 0) {
        float total = 0.0f;
        for (int w = 0; w < 8; ++w) total += warp_sum[w];
        partial[blockIdx.x] = total;
    }
}

// Rest of K5 + K6 (ngp.train.cu:443-474): the mean (sum of the 2048 partials, fixed order,
// recomputed by every CTA), threshold = min(0.01, mean), 8 cells per byte in Morton order,
// and the occupied-cell count.  Zeroes the scratch grid for the next update on the way.
__global__ void __launch_bounds__(256) bitfield_kernel(const float* __restrict__ values, const float* __restrict__ partial, uint32_t n_partial,
                                                       float* __restrict__ mean_out, uint8_t* __restrict__ bits, uint32_t* __restrict__ count,
                                                       float* __restrict__ scratch) {
    __shared__ float s_mean;
    __shared__ uint32_t s_count[8];
    if (threadIdx.x < 32) {
        float acc = 0.0f;
        for (uint32_t k = threadIdx.x; k < n_partial; k += 32) acc += partial[k];
#pragma unroll
        for (uint32_t o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xFFFFFFFFu, acc, o);
        if (threadIdx.x == 0) {
            s_mean = acc / static_cast<float>(kGridCells);
            if (blockIdx.x == 0) *mean_out = s_mean;
        }
    }
    __syncthreads();
    const float thresh  = fminf(kMinOpticalThick, s_mean);
    const uint32_t b    = blockIdx.x * 256u + threadIdx.x;  // byte index: cells 8b .. 8b+7
    const float4 lo     = reinterpret_cast<const float4*>(values)[2u * b];
    const float4 hi     = reinterpret_cast<const float4*>(values)[2u * b + 1u];
    const uint32_t byte = (lo.x > thresh ? 1u : 0u) | (lo.y > thresh ? 2u : 0u) | (lo.z > thresh ? 4u : 0u) | (lo.w > thresh ? 8u : 0u) |
                          (hi.x > thresh ? 16u : 0u) | (hi.y > thresh ? 32u : 0u) | (hi.z > thresh ? 64u : 0u) | (hi.w > thresh ? 128u : 0u);
    bits[b] = static_cast<uint8_t>(byte);
    reinterpret_cast<float4*>(scratch)[2u * b]      = make_float4(0.f, 0.f, 0.f, 0.f);
    reinterpret_cast<float4*>(scratch)[2u * b + 1u] = make_float4(0.f, 0.f, 0.f, 0.f);
    uint32_t c = __popc(byte);
#pragma unroll
    for (uint32_t o = 16; o > 0; o >>= 1) c += __shfl_down_sync(0xFFFFFFFFu, c, o);
    if ((threadIdx.x & 31u) == 0) s_count[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t total = 0;
        for (int w = 0; w < 8; ++w) total += s_count[w];
        atomicAdd(count, total);
    }
}

// ------------------------------------------------------------------------------------------
// marching
// ------------------------------------------------------------------------------------------
struct MarchParams {
    CameraSet cam;                // training rays from cameras, or
    const float* rays_in;         // explicit rays [n][6] (origin, unit direction)
    int jitter;                   // explicit rays: 1 = training PCG start jitter, 0 = half step
    uint32_t step;                // training step (PCG stream)
    const uint32_t* n_rays_dev;   // optional device-side ray count (<= n_rays)
    uint32_t n_rays;
    const uint8_t* bits;
    uint32_t* numsteps;           // [n][2] (count, base) per ray
    uint32_t* block_totals;       // per-CTA sample totals (scratch head)
    uint2* runs;                  // [n][kMaxRuns] occupied runs per ray (scratch tail)
    float* rays_out;              // training: [n][6] origin + unnormalised direction
    uint32_t* ray_indices;        // training: identity
    float* coords;                // sample records
    uint32_t sample_limit;
    uint32_t* ray_counter;
    uint32_t* sample_counter;     // total samples before the limit
    // segmented marching (rendering); unused by the other marches
    const uint32_t* list;         // entry k marches ray list[k] (null: ray k)
    const float* t_state;         // [ray] where the ray continues (null: from its start)
    const uint32_t* marched;      // [ray] samples marched before this call (null: 0)
    uint32_t cap;                 // samples per ray in this call
    float* t_out;                 // [entry] where the ray continues after this call, -1 = ended
    uint32_t* complete;           // entries [0, *complete) fitted into the sample limit
};

__device__ __forceinline__ uint32_t march_ray_count(const MarchParams& p) { return p.n_rays_dev != nullptr ? min(*p.n_rays_dev, p.n_rays) : p.n_rays; }

__device__ __forceinline__ bool setup_ray(const MarchParams& p, uint32_t i, uint32_t n, TrainRay& r) {
    if (p.rays_in == nullptr) return make_train_ray(i, n, p.step, p.cam, r);
    const float* q = p.rays_in + static_cast<uint64_t>(i) * 6u;
    r.origin       = {q[0], q[1], q[2]};
    r.dir          = {q[3], q[4], q[5]};
    r.dir_raw      = r.dir;
    float tmin;
    if (!intersect_unit_cube(r.origin, r.dir, tmin)) return false;
    if (p.jitter) {
        Pcg32 rng{kTrainSeed};
        rng.advance(static_cast<uint64_t>(p.step) << 32u);
        rng.advance(static_cast<uint64_t>(i) * kRandPerRay);
        rng.next_float();
        rng.next_float();
        r.start_t = __fmaf_rn(rng.next_float(), kConeStep, tmin);
    } else {
        r.start_t = tmin + 0.5f * kConeStep;
    }
    return true;
}

// A group of kMarchGroup lanes per ray, kRaysPerCta rays per CTA.  Count pass: per-ray step
// counts and per-CTA totals.
#ifndef NGP_MARCH_CTA
#define NGP_MARCH_CTA 256
#endif
constexpr uint32_t kCtaThreads = NGP_MARCH_CTA;
constexpr uint32_t kRaysPerCta = kCtaThreads / kMarchGroup;
// below this many threads per SM at kMarchGroup lanes per ray, training marches use 32 lanes per ray
#ifndef NGP_WIDE_MARCH_THREADS
#define NGP_WIDE_MARCH_THREADS 2048
#endif
constexpr uint32_t kWideMarchThreadsPerSm = NGP_WIDE_MARCH_THREADS;

template <uint32_t G, uint32_t RPC>
__global__ void __launch_bounds__(RPC * G) march_count_kernel(const __grid_constant__ MarchParams p) {
    __shared__ uint32_t s_steps[RPC];
    const uint32_t n    = march_ray_count(p);
    const uint32_t slot = threadIdx.x / G, g = threadIdx.x % G;
    const uint32_t i    = blockIdx.x * RPC + slot;
    TrainRay r{};
    const bool active    = i < n && setup_ray(p, i, n, r);
    uint32_t n_runs;
    const uint32_t steps = group_march_count_runs<G>(r.origin, r.dir, r.start_t, active, p.bits, p.runs + static_cast<uint64_t>(i) * kMaxRuns, n_runs);
    if (i < n && g == 0) {
        p.numsteps[2u * i]      = steps;
        p.numsteps[2u * i + 1u] = n_runs;  // read back by the write pass, then replaced by the base
        if (p.rays_out != nullptr) {
            float* o = p.rays_out + static_cast<uint64_t>(i) * 6u;
            o[0] = r.origin.x, o[1] = r.origin.y, o[2] = r.origin.z, o[3] = r.dir_raw.x, o[4] = r.dir_raw.y, o[5] = r.dir_raw.z;
        }
        if (p.ray_indices != nullptr) p.ray_indices[i] = i;
    }
    if (g == 0) s_steps[slot] = steps;
    __syncthreads();
    if (threadIdx.x < 32) {
        uint32_t total = 0;
        for (uint32_t w = threadIdx.x; w < RPC; w += 32) total += s_steps[w];
#pragma unroll
        for (uint32_t o = 16; o > 0; o >>= 1) total += __shfl_down_sync(0xFFFFFFFFu, total, o);
        if (threadIdx.x == 0) p.block_totals[blockIdx.x] = total;
    }
}

// One CTA: exclusive scan of the per-CTA totals in place; writes the grand total.
__global__ void __launch_bounds__(1024) scan_totals_kernel(uint32_t* __restrict__ totals, uint32_t n_blocks, const uint32_t* n_rays_dev,
                                                           uint32_t n_rays, uint32_t* __restrict__ grand_total, uint32_t* __restrict__ ray_counter) {
    uint32_t carry = 0;
    for (uint32_t base = 0; base < n_blocks; base += 1024u) {
        const uint32_t k = base + threadIdx.x;
        const uint32_t v = k < n_blocks ? totals[k] : 0u;
        uint32_t sum;
        const uint32_t ex = block_exclusive_scan(v, sum);
        if (k < n_blocks) totals[k] = carry + ex;
        carry += sum;
    }
    if (threadIdx.x == 0) {
        if (grand_total != nullptr) *grand_total = carry;
        if (ray_counter != nullptr) *ray_counter = n_rays_dev != nullptr ? min(*n_rays_dev, n_rays) : n_rays;
    }
}

template <uint32_t G, uint32_t RPC>
__global__ void __launch_bounds__(RPC * G) march_write_kernel(const __grid_constant__ MarchParams p) {
    __shared__ uint32_t s_base[RPC];
    __shared__ float s_stage[RPC * G * 7u];  // per warp: 32 staged sample records
    const uint32_t n    = march_ray_count(p);
    const uint32_t slot = threadIdx.x / G, g = threadIdx.x % G;
    const uint32_t i    = blockIdx.x * RPC + slot;
    // this ray's first sample: CTA base + counts of the CTA's earlier rays (exclusive scan)
    const uint32_t steps  = i < n ? p.numsteps[2u * i] : 0u;
    const uint32_t n_runs = i < n ? p.numsteps[2u * i + 1u] : 0u;
    uint32_t total;
    const uint32_t ex = block_exclusive_scan(g == 0 ? steps : 0u, total);
    if (g == 0) s_base[slot] = ex;
    __syncthreads();
    const uint32_t base = p.block_totals[blockIdx.x] + s_base[slot];
    // rays whose samples would cross the sample limit are dropped (ngp.train.cu:537-538)
    const uint32_t kept = (i < n && base + steps <= p.sample_limit) ? steps : 0u;
    if (i < n && g == 0) {
        p.numsteps[2u * i]      = kept;
        p.numsteps[2u * i + 1u] = kept ? base : 0u;
    }
    TrainRay r{};
    if (kept > 0) setup_ray(p, i, n, r);
    float* out          = p.coords + static_cast<uint64_t>(base) * 7u;
    const bool overflow = n_runs == kRunsOverflow;
    // rays with few runs expand them; the rare ray with more runs than recorded marches again
    group_expand_runs<G>(r.dir, r.origin, p.runs + static_cast<uint64_t>(i) * kMaxRuns, n_runs, kept, !overflow, out, s_stage + (threadIdx.x & ~31u) * 7u);
    group_march_write<G>(r.origin, r.dir, r.start_t, overflow ? kept : 0u, p.bits, out);
}

// Segmented marching of evaluation rays: each call marches at most `cap` further samples of the
// listed rays, continuing where the previous call stopped (see group_march_count_runs_seg).  The
// write pass keeps the entries whose samples fit under the sample limit -- a prefix of the list,
// since bases grow with the entry -- and reports its length in *complete; the first entry that
// does not fit is the one whose samples cross the limit.
__device__ __forceinline__ bool seg_ray(const MarchParams& p, uint32_t k, uint32_t n, uint32_t& i, TrainRay& r, uint32_t& limit, bool& final_limit) {
    if (k >= n) return false;
    i                    = p.list != nullptr ? p.list[k] : k;
    const uint32_t done  = p.marched != nullptr ? p.marched[i] : 0u;
    const uint32_t left  = kMarchSteps - min(done, kMarchSteps);
    limit                = min(p.cap, left);
    final_limit          = limit == left;
    if (!setup_ray(p, i, 0u, r)) return false;
    if (p.t_state != nullptr) r.start_t = p.t_state[i];
    return true;
}

__global__ void __launch_bounds__(kCtaThreads) seg_march_count_kernel(const __grid_constant__ MarchParams p) {
    __shared__ uint32_t s_steps[kRaysPerCta];
    const uint32_t n    = march_ray_count(p);
    const uint32_t slot = threadIdx.x / kMarchGroup, g = threadIdx.x % kMarchGroup;
    const uint32_t k    = blockIdx.x * kRaysPerCta + slot;
    TrainRay r{};
    uint32_t i = 0, limit = 0;
    bool final_limit  = true;
    const bool active = seg_ray(p, k, n, i, r, limit, final_limit);
    uint32_t n_runs;
    float t_after;
    const uint32_t steps = group_march_count_runs_seg(r.origin, r.dir, r.start_t, active, p.bits, limit, final_limit,
                                                      p.runs + static_cast<uint64_t>(k) * kMaxRuns, n_runs, t_after);
    if (k < n && g == 0) {
        p.numsteps[2u * k]      = steps;
        p.numsteps[2u * k + 1u] = n_runs;
        p.t_out[k]              = t_after;
    }
    if (g == 0) s_steps[slot] = steps;
    __syncthreads();
    if (threadIdx.x < 32) {
        uint32_t total = 0;
        for (uint32_t w = threadIdx.x; w < kRaysPerCta; w += 32) total += s_steps[w];
#pragma unroll
        for (uint32_t o = 16; o > 0; o >>= 1) total += __shfl_down_sync(0xFFFFFFFFu, total, o);
        if (threadIdx.x == 0) p.block_totals[blockIdx.x] = total;
    }
}

__global__ void __launch_bounds__(kCtaThreads) seg_march_write_kernel(const __grid_constant__ MarchParams p) {
    __shared__ uint32_t s_base[kRaysPerCta];
    __shared__ float s_stage[kCtaThreads * 7u];  // per warp: 32 staged sample records
    const uint32_t n      = march_ray_count(p);
    const uint32_t slot   = threadIdx.x / kMarchGroup, g = threadIdx.x % kMarchGroup;
    const uint32_t k      = blockIdx.x * kRaysPerCta + slot;
    const uint32_t steps  = k < n ? p.numsteps[2u * k] : 0u;
    const uint32_t n_runs = k < n ? p.numsteps[2u * k + 1u] : 0u;
    uint32_t total;
    const uint32_t ex = block_exclusive_scan(g == 0 ? steps : 0u, total);
    if (g == 0) s_base[slot] = ex;
    __syncthreads();
    const uint32_t base = p.block_totals[blockIdx.x] + s_base[slot];
    const bool fits     = base + steps <= p.sample_limit;
    const uint32_t kept = (k < n && fits) ? steps : 0u;
    if (k < n && g == 0) {
        p.numsteps[2u * k]      = kept;
        p.numsteps[2u * k + 1u] = kept ? base : 0u;
        if (!fits && base <= p.sample_limit) *p.complete = k;  // the one entry that crosses the limit
    }
    TrainRay r{};
    uint32_t i = 0, limit = 0;
    bool final_limit = true;
    if (kept > 0) seg_ray(p, k, n, i, r, limit, final_limit);
    float* out          = p.coords + static_cast<uint64_t>(base) * 7u;
    const bool overflow = n_runs == kRunsOverflow;
    group_expand_runs(r.dir, r.origin, p.runs + static_cast<uint64_t>(k) * kMaxRuns, n_runs, kept, !overflow, out, s_stage + (threadIdx.x & ~31u) * 7u);
    group_march_write(r.origin, r.dir, r.start_t, overflow ? kept : 0u, p.bits, out);
}

// Evaluation pixel rays (ngp.train.cu:587-614): pixel centre through the pinhole camera,
// normalised direction.  A degenerate ray gets a NaN origin, which yields no samples.
__global__ void eval_rays_kernel(const CameraSet cam, uint32_t image, uint32_t pixel_offset, uint32_t n, float* __restrict__ rays, const PixelMap map) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t gp = 0;
    float* o    = rays + static_cast<uint64_t>(i) * 6u;
    if (!map_pixel(map, pixel_offset + i, cam.width, cam.height, gp)) {
        // no pixel: a ray with no origin marches no samples
        o[0] = o[1] = o[2] = __int_as_float(0x7fc00000);
        o[3] = 1.0f, o[4] = 0.0f, o[5] = 0.0f;
        return;
    }
    const uint32_t px = gp % cam.width, py = gp / cam.width;
    const float* f    = cam.camera + static_cast<uint64_t>(image) * 12u;
    const float rx    = (static_cast<float>(px) + 0.5f - cam.principal_x) / cam.focal_x;
    const float ry    = (static_cast<float>(py) + 0.5f - cam.principal_y) / cam.focal_y;
    float3 d          = {__fmaf_rn(f[0], rx, f[3] * ry) + f[6], __fmaf_rn(f[1], rx, f[4] * ry) + f[7], __fmaf_rn(f[2], rx, f[5] * ry) + f[8]};
    if (d.x == 0.0f && d.y == 0.0f && d.z == 0.0f) d = {f[6], f[7], f[8]};
    const float len = norm3df(d.x, d.y, d.z);
    if (len == 0.0f) {
        o[0] = o[1] = o[2] = __int_as_float(0x7fc00000);
        o[3] = 1.0f, o[4] = 0.0f, o[5] = 0.0f;
        return;
    }
    o[0] = f[9], o[1] = f[10], o[2] = f[11];
    o[3] = d.x / len, o[4] = d.y / len, o[5] = d.z / len;
}

uint32_t march_blocks(uint32_t n_rays) { return (n_rays + kRaysPerCta - 1) / kRaysPerCta; }

// The wide training march (32 lanes per ray) runs kWideRaysPerCta rays per 256-thread CTA: small
// CTAs, so that an SM is not held by one CTA waiting for its longest ray.
constexpr uint32_t kWideRaysPerCta = 8;
uint32_t wide_march_blocks(uint32_t n_rays) { return (n_rays + kWideRaysPerCta - 1) / kWideRaysPerCta; }

// Scratch: per-CTA totals (room for the wide march's count), then (8-byte aligned) kMaxRuns run
// records per ray.
uint64_t march_scratch_words(uint32_t n_rays) { return ((wide_march_blocks(n_rays) + 1ull) & ~1ull) + 2ull * kMaxRuns * n_rays; }

int launch_march(MarchParams p, uint32_t* scratch, cudaStream_t s) {
    // Few rays (the first training steps march ~4096 long rays): a whole warp per ray instead of
    // kMarchGroup lanes, so that the SMs have enough warps to hide each round's latency.  The
    // positions are the sequential march's either way; only the speculation width differs.
    const bool wide = static_cast<uint64_t>(p.n_rays) * kMarchGroup < static_cast<uint64_t>(sm_count()) * kWideMarchThreadsPerSm;
    const uint32_t blocks = wide ? wide_march_blocks(p.n_rays) : march_blocks(p.n_rays);
    p.block_totals        = scratch;
    p.runs                = reinterpret_cast<uint2*>(scratch + ((wide_march_blocks(p.n_rays) + 1u) & ~1u));
    if (wide)
        march_count_kernel<32, kWideRaysPerCta><<<blocks, kWideRaysPerCta * 32u, 0, s>>>(p);
    else
        march_count_kernel<kMarchGroup, kRaysPerCta><<<blocks, kCtaThreads, 0, s>>>(p);
    NGP_TRY(check_launch("march_count_kernel"));
    scan_totals_kernel<<<1, 1024, 0, s>>>(p.block_totals, blocks, p.n_rays_dev, p.n_rays, p.sample_counter, p.ray_counter);
    NGP_TRY(check_launch("scan_totals_kernel"));
    if (wide)
        march_write_kernel<32, kWideRaysPerCta><<<blocks, kWideRaysPerCta * 32u, 0, s>>>(p);
    else
        march_write_kernel<kMarchGroup, kRaysPerCta><<<blocks, kCtaThreads, 0, s>>>(p);
    return check_launch("march_write_kernel");
}

int launch_seg_march(MarchParams p, uint32_t* scratch, cudaStream_t s) {
    const uint32_t blocks = march_blocks(p.n_rays);
    p.block_totals        = scratch;
    p.runs                = reinterpret_cast<uint2*>(scratch + ((blocks + 1u) & ~1u));
    seg_march_count_kernel<<<blocks, kCtaThreads, 0, s>>>(p);
    NGP_TRY(check_launch("seg_march_count_kernel"));
    // totals, and *complete = the entry count until an entry crosses the limit
    scan_totals_kernel<<<1, 1024, 0, s>>>(p.block_totals, blocks, p.n_rays_dev, p.n_rays, p.sample_counter, p.complete);
    NGP_TRY(check_launch("scan_totals_kernel"));
    seg_march_write_kernel<<<blocks, kCtaThreads, 0, s>>>(p);
    return check_launch("seg_march_write_kernel");
}

CameraSet camera_set(const float* camera, uint32_t frame_count, uint32_t width, uint32_t height, float fx, float fy, float cx, float cy) {
    return CameraSet{camera, frame_count, width, height, fx, fy, cx, cy};
}
bool camera_ok(const float* camera, uint32_t frame_count, uint32_t width, uint32_t height, float fx, float fy, float cx, float cy) {
    return camera != nullptr && frame_count > 0 && width > 0 && height > 0 && fx > 0.0f && fy > 0.0f && std::isfinite(cx) && std::isfinite(cy);
}

}  // namespace
}  // namespace ngp

using namespace ngp;

extern "C" uint64_t ngp_march_scratch_words(uint32_t max_rays) { return march_scratch_words(max_rays); }

extern "C" int ngp_density_grid_mark_untrained(const float* camera, uint32_t frame_count, uint32_t width, uint32_t height, float focal_x,
                                               float focal_y, float principal_x, float principal_y, float* values, void* stream) {
    clear_error();
    if (!camera_ok(camera, frame_count, width, height, focal_x, focal_y, principal_x, principal_y) || values == nullptr)
        return fail(NGP_ERR_INVALID, "mark untrained: invalid input");
    mark_untrained_kernel<<<kGridCells / 128u, 128, 0, as_stream(stream)>>>(
        values, camera_set(camera, frame_count, width, height, focal_x, focal_y, principal_x, principal_y));
    return check_launch("mark_untrained_kernel");
}

extern "C" int ngp_density_grid_samples(uint32_t n_uniform, uint32_t n_nonuniform, uint32_t ema_step, const float* values, float* coords,
                                        uint32_t* indices, void* stream) {
    clear_error();
    const uint32_t n = n_uniform + n_nonuniform;
    if (n == 0) return NGP_OK;
    if (values == nullptr || coords == nullptr || indices == nullptr) return fail(NGP_ERR_INVALID, "grid samples: null pointer");
    generate_grid_samples_kernel<<<(n + 127) / 128, 128, 0, as_stream(stream)>>>(n_uniform, n_nonuniform, ema_step, values, coords, indices);
    return check_launch("generate_grid_samples_kernel");
}

extern "C" int ngp_density_grid_samples_cell_order(uint32_t n_uniform, uint32_t n_nonuniform, uint32_t ema_step, const float* values, float* coords,
                                                   uint32_t* indices, uint32_t* counter, void* stream) {
    clear_error();
    const uint32_t n = n_uniform + n_nonuniform;
    if (n == 0) return NGP_OK;
    if (values == nullptr || coords == nullptr || indices == nullptr) return fail(NGP_ERR_INVALID, "grid samples: null pointer");
    if (n_uniform > kGridCells || n_nonuniform > kGridCells) return fail(NGP_ERR_INVALID, "grid samples (cell order): at most 2^21 samples per set");
    const bool direct = n_uniform == kGridCells && n_nonuniform == 0;
    if (!direct && counter == nullptr) return fail(NGP_ERR_INVALID, "grid samples (cell order): counter needed unless all 2^21 samples are uniform");
    const cudaStream_t s = as_stream(stream);
    if (!direct) NGP_TRY(check_cuda(cudaMemsetAsync(counter, 0, sizeof(uint32_t), s), "grid samples: clear counter"));
    // the sets' streams before the per-sample jump: PCG32(1337) advanced by (2 ema_step + phase + 1) << 32
    Pcg32 u{kTrainSeed}, v{kTrainSeed};
    u.advance((static_cast<uint64_t>(ema_step) * 2ull + 1ull) << 32u);
    v.advance((static_cast<uint64_t>(ema_step) * 2ull + 2ull) << 32u);
    generate_grid_samples_ordered_kernel<<<kGridCells / 256u, 256, 0, s>>>(n_uniform, n_nonuniform, ema_step, u.state, v.state, values, coords, indices,
                                                                           direct ? nullptr : counter);
    return check_launch("generate_grid_samples_ordered_kernel");
}

extern "C" int ngp_density_grid_splat(uint32_t n, const uint32_t* indices, const uint16_t* density, float* scratch, void* stream) {
    clear_error();
    if (n == 0) return NGP_OK;
    if (indices == nullptr || density == nullptr || scratch == nullptr) return fail(NGP_ERR_INVALID, "grid splat: null pointer");
    splat_kernel<<<(n + 127) / 128, 128, 0, as_stream(stream)>>>(n, indices, reinterpret_cast<const __half*>(density), scratch);
    return check_launch("splat_kernel");
}

extern "C" uint32_t ngp_density_grid_partials(void) { return kGridCells / 1024u; }

extern "C" int ngp_density_grid_update(float* values, float* scratch, float decay, float* partial, float* mean, uint8_t* bitfield,
                                       uint32_t* occupied_count, void* stream) {
    clear_error();
    if (values == nullptr || scratch == nullptr || partial == nullptr || mean == nullptr || bitfield == nullptr || occupied_count == nullptr)
        return fail(NGP_ERR_INVALID, "grid update: null pointer");
    const cudaStream_t s = as_stream(stream);
    ema_partial_kernel<<<kGridCells / 1024u, 256, 0, s>>>(scratch, values, decay, partial);
    NGP_TRY(check_launch("ema_partial_kernel"));
    NGP_TRY(check_cuda(cudaMemsetAsync(occupied_count, 0, sizeof(uint32_t), s), "grid update: clear count"));
    bitfield_kernel<<<kGridCells / 8u / 256u, 256, 0, s>>>(values, partial, kGridCells / 1024u, mean, bitfield, occupied_count, scratch);
    return check_launch("bitfield_kernel");
}

extern "C" int ngp_march_training_rays(const float* camera, uint32_t frame_count, uint32_t width, uint32_t height, float focal_x, float focal_y,
                                       float principal_x, float principal_y, uint32_t step, uint32_t rays_per_batch,
                                       const uint32_t* rays_per_batch_dev, uint32_t sample_limit, const uint8_t* bitfield, float* coords,
                                       float* rays, uint32_t* ray_indices, uint32_t* numsteps, uint32_t* scratch, uint32_t* ray_counter,
                                       uint32_t* sample_counter, void* stream) {
    clear_error();
    if (rays_per_batch == 0) return NGP_OK;
    if (!camera_ok(camera, frame_count, width, height, focal_x, focal_y, principal_x, principal_y) || bitfield == nullptr || coords == nullptr ||
        numsteps == nullptr || scratch == nullptr || sample_limit == 0)
        return fail(NGP_ERR_INVALID, "march training rays: invalid input");
    MarchParams p{};
    p.cam            = camera_set(camera, frame_count, width, height, focal_x, focal_y, principal_x, principal_y);
    p.step           = step;
    p.n_rays_dev     = rays_per_batch_dev;
    p.n_rays         = rays_per_batch;
    p.bits           = bitfield;
    p.numsteps       = numsteps;
    p.rays_out       = rays;
    p.ray_indices    = ray_indices;
    p.coords         = coords;
    p.sample_limit   = sample_limit;
    p.ray_counter    = ray_counter;
    p.sample_counter = sample_counter;
    return launch_march(p, scratch, as_stream(stream));
}

extern "C" int ngp_march_rays(uint32_t n_rays, const float* rays, int jitter, uint32_t step, const uint8_t* bitfield, uint32_t sample_limit,
                              float* coords, uint32_t* numsteps, uint32_t* scratch, uint32_t* sample_counter, void* stream) {
    clear_error();
    if (n_rays == 0) return NGP_OK;
    if (rays == nullptr || bitfield == nullptr || coords == nullptr || numsteps == nullptr || scratch == nullptr || sample_limit == 0)
        return fail(NGP_ERR_INVALID, "march rays: invalid input");
    MarchParams p{};
    p.n_rays         = n_rays;
    p.rays_in        = rays;
    p.jitter         = jitter;
    p.step           = step;
    p.bits           = bitfield;
    p.numsteps       = numsteps;
    p.coords         = coords;
    p.sample_limit   = sample_limit;
    p.sample_counter = sample_counter;
    return launch_march(p, scratch, as_stream(stream));
}

extern "C" int ngp_march_rays_segment(uint32_t max_entries, const uint32_t* n_entries, const uint32_t* list, const float* rays,
                                      const uint8_t* bitfield, const float* t_state, const uint32_t* marched, uint32_t cap, uint32_t sample_limit,
                                      float* coords, uint32_t* numsteps, float* t_out, uint32_t* scratch, uint32_t* counters, void* stream) {
    clear_error();
    if (max_entries == 0) return NGP_OK;
    if (rays == nullptr || bitfield == nullptr || coords == nullptr || numsteps == nullptr || t_out == nullptr || scratch == nullptr ||
        counters == nullptr || sample_limit == 0 || cap == 0 || (t_state == nullptr) != (marched == nullptr))
        return fail(NGP_ERR_INVALID, "segment march: invalid input");
    // the first segment starts every ray: all of it must fit (later segments keep what does not)
    if (t_state == nullptr && static_cast<uint64_t>(cap) * max_entries > sample_limit)
        return fail(NGP_ERR_INVALID, "segment march: the first segment (cap x rays) must fit the sample limit");
    MarchParams p{};
    p.n_rays         = max_entries;
    p.n_rays_dev     = n_entries;
    p.rays_in        = rays;
    p.jitter         = 0;
    p.bits           = bitfield;
    p.numsteps       = numsteps;
    p.coords         = coords;
    p.sample_limit   = sample_limit;
    p.sample_counter = counters;
    p.complete       = counters + 1;
    p.list           = list;
    p.t_state        = t_state;
    p.marched        = marched;
    p.cap            = cap;
    p.t_out          = t_out;
    return launch_seg_march(p, scratch, as_stream(stream));
}

extern "C" int ngp_make_eval_rays(const float* camera, uint32_t image, uint32_t width, uint32_t height, float focal_x, float focal_y,
                                  float principal_x, float principal_y, uint32_t pixel_offset, uint32_t n, float* rays, void* stream) {
    clear_error();
    if (n == 0) return NGP_OK;
    if (!camera_ok(camera, image + 1u, width, height, focal_x, focal_y, principal_x, principal_y) || rays == nullptr)
        return fail(NGP_ERR_INVALID, "eval rays: invalid input");
    eval_rays_kernel<<<(n + 127) / 128, 128, 0, as_stream(stream)>>>(camera_set(camera, image + 1u, width, height, focal_x, focal_y, principal_x, principal_y),
                                                                    image, pixel_offset, n, rays, PixelMap{0u, 0u, 0u});
    return check_launch("eval_rays_kernel");
}

extern "C" int ngp_make_eval_rays_tiles(const float* camera, uint32_t image, uint32_t width, uint32_t height, float focal_x, float focal_y,
                                        float principal_x, float principal_y, uint32_t first_tile, uint32_t tile_stride, uint32_t slot_offset,
                                        uint32_t n, float* rays, void* stream) {
    clear_error();
    if (n == 0) return NGP_OK;
    if (!camera_ok(camera, image + 1u, width, height, focal_x, focal_y, principal_x, principal_y) || rays == nullptr || tile_stride == 0)
        return fail(NGP_ERR_INVALID, "eval rays (tiles): invalid input");
    const PixelMap map{(width + kTileSide - 1u) / kTileSide, first_tile, tile_stride};
    eval_rays_kernel<<<(n + 127) / 128, 128, 0, as_stream(stream)>>>(camera_set(camera, image + 1u, width, height, focal_x, focal_y, principal_x, principal_y),
                                                                    image, slot_offset, n, rays, map);
    return check_launch("eval_rays_kernel");
}
