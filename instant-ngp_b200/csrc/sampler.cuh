// Device helpers shared by the occupancy grid, ray marching and compositing kernels.
//
// The geometric helpers restate the reference's (ngp.train.cu:195-308).  Their floating-point
// expressions keep the reference's evaluation order; where the reference source has an a*b+c
// form that the compiler contracts into one fused multiply-add, the fused form is written out
// explicitly (__fmaf_rn), so sample positions are identical bit for bit.
#pragma once

#include "common.cuh"

namespace ngp {

constexpr uint32_t kGridSize      = 128u;
constexpr uint32_t kGridCells     = kGridSize * kGridSize * kGridSize;
constexpr uint32_t kMarchSteps    = 1024u;
// rows of the compacted training buffers: the batch plus one whole ray straddling its end
constexpr uint32_t kCompactedRows = (1u << 18) + kMarchSteps;
constexpr float kConeStep         = 1.73205080757f / 1024.0f;  // sqrt(3) / NERF_STEPS
constexpr uint32_t kRandPerRay    = 16u;                       // MAX_RANDOM_SAMPLES_PER_RAY
constexpr float kMinOpticalThick  = 0.01f;
constexpr float kTransmittanceEps = 1e-4f;
constexpr uint32_t kNetworkBatch  = 1u << 18;                  // NETWORK_BATCH_SIZE
constexpr uint32_t kMaxSamples    = kNetworkBatch * 16u;       // MAX_SAMPLES
constexpr uint32_t kBatchGranule  = 128u;
constexpr float kLossScale        = 128.0f;

// 3-bit interleave of a 7-bit coordinate (Morton order of the 128^3 grid).
__host__ __device__ __forceinline__ uint32_t morton_spread(uint32_t v) {
    v = (v * 0x00010001u) & 0xFF0000FFu;
    v = (v * 0x00000101u) & 0x0F00F00Fu;
    v = (v * 0x00000011u) & 0xC30C30C3u;
    v = (v * 0x00000005u) & 0x49249249u;
    return v;
}
__host__ __device__ __forceinline__ uint32_t morton_compact(uint32_t v) {
    v &= 0x49249249u;
    v = (v | (v >> 2u)) & 0xC30C30C3u;
    v = (v | (v >> 4u)) & 0x0F00F00Fu;
    v = (v | (v >> 8u)) & 0xFF0000FFu;
    v = (v | (v >> 16u)) & 0x0000FFFFu;
    return v;
}

// K2's cell hash (ngp.train.cu:383-424): sample i of a set of `count` (try j) takes cell
// ((i + ema_step * count) * 56924617 + j * 19349663 + 96925573) mod 2^21.  The multiplier is odd,
// so with j = 0 this is a bijection of [0, 2^21) (inverse multiplier 53369).
constexpr uint32_t kGridHashMul    = 56924617u;
constexpr uint32_t kGridHashMulInv = 53369u;  // inverse of 56924617 modulo 2^21
constexpr uint32_t kGridHashAdd    = 96925573u;

// Position and cell of grid sample i of its set (K2's body): up to 10 hashed tries for a cell
// whose value exceeds `thresh`, then the cell corner plus three PCG32 draws of sample i's stream
// (the set's base state advanced by 4 i steps; jm / jp: the 2^k jump table in shared memory).
__device__ __forceinline__ void grid_sample_position(uint32_t i, uint32_t count, uint32_t ema_step, float thresh, uint64_t base_state,
                                                     const uint64_t* __restrict__ jm, const uint64_t* __restrict__ jp,
                                                     const float* __restrict__ values, float (&pos)[3], uint32_t& idx) {
    idx = 0;
    for (uint32_t j = 0; j < 10; ++j) {
        idx = static_cast<uint32_t>(((static_cast<uint64_t>(i) + static_cast<uint64_t>(ema_step) * count) * kGridHashMul +
                                     static_cast<uint64_t>(j) * 19349663ull + kGridHashAdd) %
                                    kGridCells);
        if (values[idx] > thresh) break;
    }
    uint64_t state = base_state;
    for (uint64_t delta = static_cast<uint64_t>(i) * 4ull; delta != 0u; delta &= delta - 1u) {
        const int k = __ffsll(static_cast<long long>(delta)) - 1;
        state       = jm[k] * state + jp[k];
    }
    Pcg32 rng{0u};
    rng.state = state;
    rng.inc   = 3u;
    const uint32_t x = morton_compact(idx), y = morton_compact(idx >> 1), z = morton_compact(idx >> 2);
    pos[0] = (static_cast<float>(x) + rng.next_float()) / 128.0f;
    pos[1] = (static_cast<float>(y) + rng.next_float()) / 128.0f;
    pos[2] = (static_cast<float>(z) + rng.next_float()) / 128.0f;
}

__device__ __forceinline__ bool inside_unit_cube(float3 p) {
    return p.x >= 0.0f && p.x <= 1.0f && p.y >= 0.0f && p.y <= 1.0f && p.z >= 0.0f && p.z <= 1.0f;
}

// Slab test against [0,1]^3; out_tmin = max(entry, 0).
__device__ __forceinline__ bool intersect_unit_cube(float3 o, float3 d, float& out_tmin) {
    const float3 inv = {1.0f / d.x, 1.0f / d.y, 1.0f / d.z};
    const float3 t0  = {-o.x * inv.x, -o.y * inv.y, -o.z * inv.z};
    const float3 t1  = {(1.0f - o.x) * inv.x, (1.0f - o.y) * inv.y, (1.0f - o.z) * inv.z};
    const float tmin = fmaxf(fmaxf(fminf(t0.x, t1.x), fminf(t0.y, t1.y)), fminf(t0.z, t1.z));
    const float tmax = fminf(fminf(fmaxf(t0.x, t1.x), fmaxf(t0.y, t1.y)), fmaxf(t0.z, t1.z));
    out_tmin         = fmaxf(tmin, 0.0f);
    return tmax >= out_tmin;
}

__device__ __forceinline__ bool occupied(float3 p, const uint8_t* __restrict__ bits) {
    const int x = static_cast<int>(p.x * 128.0f), y = static_cast<int>(p.y * 128.0f), z = static_cast<int>(p.z * 128.0f);
    if (x < 0 || x >= 128 || y < 0 || y >= 128 || z < 0 || z >= 128) return false;
    const uint32_t idx = morton_spread(static_cast<uint32_t>(x)) | (morton_spread(static_cast<uint32_t>(y)) << 1u) |
                         (morton_spread(static_cast<uint32_t>(z)) << 2u);
    return (__ldg(bits + idx / 8u) >> (idx % 8u)) & 1u;
}

// Jump to the next occupancy-voxel boundary, quantised to whole cone steps.
__device__ __forceinline__ float skip_empty_voxel(float t, float3 pos, float3 dir, float3 inv_dir) {
    const float3 p = {(pos.x - 0.5f) * 128.0f, (pos.y - 0.5f) * 128.0f, (pos.z - 0.5f) * 128.0f};
    const float tx = (floorf(__fmaf_rn(0.5f, copysignf(1.0f, dir.x), p.x + 0.5f)) - p.x) * inv_dir.x;
    const float ty = (floorf(__fmaf_rn(0.5f, copysignf(1.0f, dir.y), p.y + 0.5f)) - p.y) * inv_dir.y;
    const float tz = (floorf(__fmaf_rn(0.5f, copysignf(1.0f, dir.z), p.z + 0.5f)) - p.z) * inv_dir.z;
    const float t_target = t + fmaxf(fminf(fminf(tx, ty), tz) / 128.0f, 0.0f);
    return __fmaf_rn(ceilf(fmaxf((t_target - t) / kConeStep, 0.5f)), kConeStep, t);
}

// t after k sequential additions of kConeStep (((t + dt) + dt) + ...), the march's step rule.
// Inside one binade [2^E, 2^(E+1)) every addition to a value on that binade's grid (spacing u)
// adds the same rounded increment d = round(dt / u) * u (round to nearest; a tie, where the
// rounding would depend on the parity, is excluded), so while every partial sum stays below
// 2^(E+1) the k-th value is exactly t + k * d, one fused multiply-add.  Otherwise (the sum
// crosses a power of two, or t is tiny) the additions run one by one.  Bit-identical to the loop.
// (the plain loop: cheaper for the few additions of a narrow group)
__device__ __forceinline__ float cone_steps_loop(float t, uint32_t k) {
    for (uint32_t j = 0; j < k; ++j) t += kConeStep;
    return t;
}

__device__ __forceinline__ float cone_steps(float t, uint32_t k) {
    const uint32_t e = __float_as_uint(t) & 0x7F800000u;
    if (k != 0 && t > 0.0f && e >= (24u << 23) && e < 0x7F000000u) {
        const float u   = __uint_as_float(e - (23u << 23));  // 2^(E-23)
        const float top = __uint_as_float(e + (1u << 23));   // 2^(E+1)
        const float m   = kConeStep / u;                      // exact: u is a power of two
        const float mf  = floorf(m), fr = m - mf;
        if (fr != 0.5f && m < 8388608.0f) {
            const float d    = (fr > 0.5f ? mf + 1.0f : mf) * u;
            const float last = __fmaf_rn(static_cast<float>(k), d, t);
            if (last + u <= top) return last;
        }
    }
    for (uint32_t j = 0; j < k; ++j) t += kConeStep;
    return t;
}

__device__ __forceinline__ float3 ray_point(float3 o, float3 d, float t) {
    return {__fmaf_rn(d.x, t, o.x), __fmaf_rn(d.y, t, o.y), __fmaf_rn(d.z, t, o.z)};
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

__device__ __forceinline__ float srgb_to_linear_c(float v) { return v <= 0.04045f ? v / 12.92f : powf((v + 0.055f) / 1.055f, 2.4f); }
__device__ __forceinline__ float linear_to_srgb_c(float v) { return v < 0.0031308f ? 12.92f * v : __fmaf_rn(1.055f, powf(v, 0.41666f), -0.055f); }

// Premultiplied linear RGBA of an RGBA8 sRGB texel (ngp.train.cu:280-293).
__device__ __forceinline__ float4 read_texel(uint32_t px, uint32_t py, uint32_t image, uint32_t width, uint32_t height,
                                             const uint8_t* __restrict__ pixels) {
    const uint32_t rgba = __ldg(reinterpret_cast<const uint32_t*>(pixels) + (px + static_cast<uint64_t>(py) * width +
                                                                            static_cast<uint64_t>(image) * width * height));
    float4 r = {static_cast<float>(rgba & 0xFFu) * (1.0f / 255.0f), static_cast<float>((rgba >> 8) & 0xFFu) * (1.0f / 255.0f),
                static_cast<float>((rgba >> 16) & 0xFFu) * (1.0f / 255.0f), static_cast<float>(rgba >> 24) * (1.0f / 255.0f)};
    r.x = srgb_to_linear_c(r.x) * r.w;
    r.y = srgb_to_linear_c(r.y) * r.w;
    r.z = srgb_to_linear_c(r.z) * r.w;
    return r;
}

// Pixel enumeration of an evaluation / render: linear (slot j = pixel j, tiles_x = 0), or a set
// of 64 x 64 tiles -- tiles first, first + stride, ... of the image's row-major tile grid
// (tiles_x tiles per row) -- with slot j = pixel (j & 4095) of the set's tile j >> 12, row-major
// inside the tile.  Slots that fall outside the image (the partial tiles at the right and bottom
// edges) map to no pixel.
struct PixelMap {
    uint32_t tiles_x, first, stride;
};

constexpr uint32_t kTileSide = 64u, kTilePixels = kTileSide * kTileSide;

__device__ __forceinline__ bool map_pixel(const PixelMap& m, uint32_t j, uint32_t width, uint32_t height, uint32_t& gp) {
    if (m.tiles_x == 0) {
        gp = j;
        return j < width * height;
    }
    const uint32_t tile = m.first + (j / kTilePixels) * m.stride, q = j % kTilePixels;
    const uint32_t x = (tile % m.tiles_x) * kTileSide + q % kTileSide, y = (tile / m.tiles_x) * kTileSide + q / kTileSide;
    gp = y * width + x;
    return x < width && y < height;
}

// Camera frames: 12 floats per frame = three axis columns and the origin (ngp.dataset.cpp:63).
struct CameraSet {
    const float* camera;
    uint32_t frame_count, width, height;
    float focal_x, focal_y, principal_x, principal_y;
};

// Training ray i of a batch (ngp.train.cu:480-517): image by stratified index, pixel from the
// step's PCG32 stream (snapped to the pixel centre), direction through the pinhole camera.
// Returns false when the ray misses the unit cube.
struct TrainRay {
    float3 origin, dir_raw, dir;
    float start_t;
};

__device__ __forceinline__ bool make_train_ray(uint32_t i, uint32_t rays_per_batch, uint32_t step, const CameraSet& cam, TrainRay& r) {
    const uint32_t image = static_cast<uint32_t>((static_cast<uint64_t>(i) * cam.frame_count) / rays_per_batch) % cam.frame_count;
    const float* f       = cam.camera + static_cast<uint64_t>(image) * 12u;
    Pcg32 rng{kTrainSeed};
    rng.advance(static_cast<uint64_t>(step) << 32u);
    rng.advance(static_cast<uint64_t>(i) * kRandPerRay);
    float u = rng.next_float();
    float v = rng.next_float();
    const uint32_t px = min(static_cast<uint32_t>(u * static_cast<float>(cam.width)), cam.width - 1u);
    const uint32_t py = min(static_cast<uint32_t>(v * static_cast<float>(cam.height)), cam.height - 1u);
    u                 = (static_cast<float>(px) + 0.5f) / static_cast<float>(cam.width);
    v                 = (static_cast<float>(py) + 0.5f) / static_cast<float>(cam.height);
    const float ray_x = __fmaf_rn(u, static_cast<float>(cam.width), -cam.principal_x) / cam.focal_x;
    const float ray_y = __fmaf_rn(v, static_cast<float>(cam.height), -cam.principal_y) / cam.focal_y;
    r.origin          = {f[9], f[10], f[11]};
    r.dir_raw = {__fmaf_rn(f[0], ray_x, f[3] * ray_y) + f[6], __fmaf_rn(f[1], ray_x, f[4] * ray_y) + f[7],
                 __fmaf_rn(f[2], ray_x, f[5] * ray_y) + f[8]};
    if (r.dir_raw.x == 0.0f && r.dir_raw.y == 0.0f && r.dir_raw.z == 0.0f) r.dir_raw = {f[6], f[7], f[8]};
    const float len = norm3df(r.dir_raw.x, r.dir_raw.y, r.dir_raw.z);
    if (len == 0.0f) return false;
    r.dir = {r.dir_raw.x / len, r.dir_raw.y / len, r.dir_raw.z / len};
    float tmin;
    if (!intersect_unit_cube(r.origin, r.dir, tmin)) return false;
    r.start_t = __fmaf_rn(rng.next_float(), kConeStep, tmin);
    return true;
}

// ---- block-wide exclusive scan of one uint32 per thread (blockDim.x multiple of 32, <= 1024) ----
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t& total) {
    __shared__ uint32_t warp_sums[32];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (uint32_t o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31u) warp_sums[warp] = x;
    __syncthreads();
    const uint32_t n_warps = blockDim.x >> 5;
    if (warp == 0) {
        uint32_t w = lane < n_warps ? warp_sums[lane] : 0u;
#pragma unroll
        for (uint32_t o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < n_warps) warp_sums[lane] = w;
    }
    __syncthreads();
    total                 = warp_sums[n_warps - 1];
    const uint32_t before = warp == 0 ? 0u : warp_sums[warp - 1];
    __syncthreads();
    return before + x - v;
}

}  // namespace ngp

namespace ngp {

// ---- group-cooperative marching --------------------------------------------------------------
// A group of G adjacent lanes marches one ray (32 / G rays per warp).  Each round the group
// speculates on the occupancy of the next G positions of the sequential march and keeps the
// prefix whose speculation held, so every accepted position is computed by exactly the
// sequential march's float operations (results are bit-identical to a one-thread loop that
// steps by dt on occupied cells and skips empty voxels, as the reference's K7 does):
//  * run mode (the last position seen was occupied): lane g takes t_g = ((t + dt) + dt) ...
//    (g sequential additions), i.e. it assumes the lanes before it were occupied.  Lanes before
//    the first unoccupied lane f are samples; lane f's position decides the skip (or the end).
//  * skip mode (the last position seen was empty): lane g applies g successive empty-voxel skips
//    to t, i.e. it assumes the lanes before it were inside the grid and empty.  The first lane f
//    that is occupied is a sample (then run mode continues at t_f + dt); an outside lane ends the
//    ray; with all G empty the march continues from the skip after lane G-1.
// Up to G occupied steps or G empty voxels are resolved per round.
#ifndef NGP_MARCH_GROUP
#define NGP_MARCH_GROUP 8
#endif
#ifndef NGP_MARCH_SKIP_WIDTH
#define NGP_MARCH_SKIP_WIDTH 4  // empty voxels speculated per skip round (measured: 2, 3, 4, 8, 16)
#endif
#ifndef NGP_MARCH_SKIP_SPEC
#define NGP_MARCH_SKIP_SPEC 1  // 0: empty voxels are skipped one per round
#endif
constexpr uint32_t kMarchGroup = NGP_MARCH_GROUP;

struct GroupMarch {
    float3 o, d, inv;
    float t;
    uint32_t n;
    bool done;
    bool skip;  // next round speculates empty voxels
};

__device__ __forceinline__ void group_march_begin(GroupMarch& m, float3 o, float3 d, float start_t, bool active) {
    m.o = o, m.d = d, m.inv = {1.0f / d.x, 1.0f / d.y, 1.0f / d.z}, m.t = start_t, m.n = 0, m.done = !active, m.skip = false;
}

// Result of one round for the calling lane's group.
struct MarchRound {
    uint32_t k;      // samples emitted (uniform in the group)
    float first_t;   // t of the first emitted sample
    bool emit;       // this lane's position is an emitted sample ...
    uint32_t slot;   // ... the slot-th of this round
    float3 pos;      // this lane's position
    float t;         // this lane's t
    bool cont;       // the next round's first position directly follows the last emitted sample
};

// One round for every group of the warp (all 32 lanes call it together); G lanes per ray.
template <uint32_t G = kMarchGroup>
__device__ __forceinline__ MarchRound group_march_round(GroupMarch& m, const uint8_t* __restrict__ bits, uint32_t limit) {
    const uint32_t lane     = threadIdx.x & 31u;
    const uint32_t g        = lane % G;
    const uint32_t group_lo = lane - g;
    const bool skip_mode    = NGP_MARCH_SKIP_SPEC && m.skip;
    float tk                = m.t;
    if (skip_mode) {
        // a group speculates on kSkipWidth voxels only (lanes past it repeat the last one's
        // position, so they never stop first): empty stretches are mostly short, and every
        // lane's chain of skips costs the warp its longest chain
        constexpr uint32_t kSkipWidth = G > NGP_MARCH_SKIP_WIDTH ? NGP_MARCH_SKIP_WIDTH : G;
        const uint32_t gs = g < kSkipWidth ? g : kSkipWidth - 1u;
        for (uint32_t j = 0; j < gs; ++j) tk = skip_empty_voxel(tk, ray_point(m.o, m.d, tk), m.d, m.inv);
    } else {
        tk = G > 8u ? cone_steps(tk, g) : cone_steps_loop(tk, g);
    }
    MarchRound r;
    r.pos                = ray_point(m.o, m.d, tk);
    r.t                  = tk;
    const bool ins       = !m.done && inside_unit_cube(r.pos);
    const bool oc        = ins && occupied(r.pos, bits);
    const bool stop_here = skip_mode ? (!ins || oc) : !oc;
    const uint32_t stop  = (__ballot_sync(0xFFFFFFFFu, stop_here) >> group_lo) & (G == 32u ? 0xFFFFFFFFu : ((1u << G) - 1u));
    const uint32_t f     = stop ? static_cast<uint32_t>(__ffs(stop)) - 1u : G;
    const uint32_t fl    = group_lo + (f < G ? f : G - 1u);
    const float next     = skip_empty_voxel(tk, r.pos, m.d, m.inv);
    const float f_t      = __shfl_sync(0xFFFFFFFFu, tk, fl);
    const bool f_inside  = __shfl_sync(0xFFFFFFFFu, ins, fl);
    const float f_next   = __shfl_sync(0xFFFFFFFFu, next, fl);
    const float t_last   = __shfl_sync(0xFFFFFFFFu, tk, group_lo + G - 1u);
    r.k = 0, r.first_t = 0.0f, r.emit = false, r.slot = 0, r.cont = false;
    if (m.done) return r;
    const uint32_t room = limit - m.n;
    if (skip_mode) {
        if (f == G) {
            m.t = f_next;  // G empty voxels: lane G-1's skip
        } else if (!f_inside) {
            m.done = true;
        } else {
            r.k = 1, r.first_t = f_t, r.emit = g == f, r.slot = 0;
            m.n += 1;
            m.t    = f_t + kConeStep;
            m.skip = false;
            if (m.n >= limit) m.done = true;
        }
    } else {
        r.k = f < room ? f : room;
        r.first_t = m.t, r.emit = g < r.k, r.slot = g;
        m.n += r.k;
        if (m.n >= limit) {
            m.done = true;
        } else if (f == G) {
            m.t = t_last + kConeStep;
        } else if (!f_inside) {
            m.done = true;
        } else {
            m.t    = f_next;
            m.skip = NGP_MARCH_SKIP_SPEC;
        }
    }
    r.cont = r.k > 0 && !m.done && !m.skip;
    return r;
}

// Writes exactly `n` records (n = this ray's count) starting at `out`; n = 0 for inactive groups.
template <uint32_t G = kMarchGroup>
__device__ __forceinline__ void group_march_write(float3 o, float3 d, float start_t, uint32_t n, const uint8_t* __restrict__ bits,
                                                  float* __restrict__ out) {
    const float3 w3 = {(d.x + 1.0f) * 0.5f, (d.y + 1.0f) * 0.5f, (d.z + 1.0f) * 0.5f};
    GroupMarch m;
    group_march_begin(m, o, d, start_t, n > 0);
    while (__any_sync(0xFFFFFFFFu, !m.done)) {
        const uint32_t before = m.n;
        const MarchRound r    = group_march_round<G>(m, bits, n);
        if (r.emit) {
            float* c = out + static_cast<uint64_t>(before + r.slot) * 7u;
            c[0] = r.pos.x, c[1] = r.pos.y, c[2] = r.pos.z, c[3] = kConeStep, c[4] = w3.x, c[5] = w3.y, c[6] = w3.z;
        }
    }
}

// ---- occupied runs ----------------------------------------------------------------------------
// The count pass records each ray's runs of consecutive occupied cone steps (the t of the run's
// first sample and its length).  The write pass then expands the runs with the same sequential
// t additions instead of marching through empty space a second time; a ray with more than
// kMaxRuns runs is marched again instead.
constexpr uint32_t kMaxRuns      = 48u;
constexpr uint32_t kRunsOverflow = 0xFFFFFFFFu;

// Sample count of this group's ray (all lanes of the warp call it; inactive groups pass
// active=false); its runs go to `runs`, their number (or kRunsOverflow) to n_runs.
template <uint32_t G = kMarchGroup>
__device__ __forceinline__ uint32_t group_march_count_runs(float3 o, float3 d, float start_t, bool active, const uint8_t* __restrict__ bits,
                                                           uint2* __restrict__ runs, uint32_t& n_runs) {
    const uint32_t g = (threadIdx.x & 31u) % G;
    GroupMarch m;
    group_march_begin(m, o, d, start_t, active);
    float run_t0   = 0.0f;
    uint32_t run_n = 0;
    n_runs         = 0;
    while (__any_sync(0xFFFFFFFFu, !m.done)) {
        const MarchRound r = group_march_round<G>(m, bits, kMarchSteps);
        if (r.k > 0) {
            if (run_n == 0) run_t0 = r.first_t;
            run_n += r.k;
        }
        if (!r.cont && run_n > 0) {
            if (n_runs < kMaxRuns && g == 0) runs[n_runs] = make_uint2(__float_as_uint(run_t0), run_n);
            ++n_runs;
            run_n = 0;
        }
    }
    if (n_runs > kMaxRuns) n_runs = kRunsOverflow;
    return m.n;
}

// Segmented marching (rendering): the same count pass with a per-call sample limit, which also
// returns where the sequential march would continue.  After a sample at t the sequential march
// evaluates t + dt next, so a march started at `t_after` in run mode continues the sequence
// exactly.  `t_after` is -1 when the ray has ended (it left the grid, or `limit` was the ray's
// remaining step allowance) and nothing follows.
__device__ __forceinline__ uint32_t group_march_count_runs_seg(float3 o, float3 d, float start_t, bool active, const uint8_t* __restrict__ bits,
                                                               uint32_t limit, bool limit_is_final, uint2* __restrict__ runs, uint32_t& n_runs,
                                                               float& t_after) {
    const uint32_t lane     = threadIdx.x & 31u;
    const uint32_t g        = lane % kMarchGroup;
    const uint32_t group_lo = lane - g;
    GroupMarch m;
    group_march_begin(m, o, d, start_t, active && limit > 0);
    float run_t0   = 0.0f;
    uint32_t run_n = 0;
    float t_last   = 0.0f;
    n_runs         = 0;
    while (__any_sync(0xFFFFFFFFu, !m.done)) {
        const MarchRound r = group_march_round(m, bits, limit);
        // t of the round's last emitted sample, from the lane that emitted it
        const bool is_last  = r.emit && r.slot + 1u == r.k;
        const uint32_t lb   = (__ballot_sync(0xFFFFFFFFu, is_last) >> group_lo) & ((1u << kMarchGroup) - 1u);
        const float t_emit  = __shfl_sync(0xFFFFFFFFu, r.t, group_lo + (lb ? static_cast<uint32_t>(__ffs(lb)) - 1u : 0u));
        if (r.k > 0) {
            t_last = t_emit;
            if (run_n == 0) run_t0 = r.first_t;
            run_n += r.k;
        }
        if (!r.cont && run_n > 0) {
            if (n_runs < kMaxRuns && g == 0) runs[n_runs] = make_uint2(__float_as_uint(run_t0), run_n);
            ++n_runs;
            run_n = 0;
        }
    }
    if (n_runs > kMaxRuns) n_runs = kRunsOverflow;
    // the march stopped at the limit (not at the grid's edge) and the limit was only this call's
    t_after = (active && limit > 0 && m.n >= limit && !limit_is_final) ? t_last + kConeStep : -1.0f;
    return m.n;
}

// Expand this group's runs into `n` sample records at `out` (active = the ray's runs are valid).
// Each round the group's lanes compute up to kMarchGroup consecutive records, stage them in this
// warp's 32 x 7 floats of shared memory (`stage`), and copy them out as consecutive floats, so a
// store instruction writes whole 32-byte sectors instead of one float every 28 bytes.
template <uint32_t G = kMarchGroup>
__device__ __forceinline__ void group_expand_runs(float3 d_unit, float3 o, const uint2* __restrict__ runs, uint32_t n_runs, uint32_t n,
                                                  bool active, float* __restrict__ out, float* __restrict__ stage) {
    const float3 w3         = {(d_unit.x + 1.0f) * 0.5f, (d_unit.y + 1.0f) * 0.5f, (d_unit.z + 1.0f) * 0.5f};
    const uint32_t lane     = threadIdx.x & 31u;
    const uint32_t g        = lane % G;
    const uint32_t group_lo = lane - g;
    uint32_t r = 0, in_run = 0, written = 0, cnt = 0;
    float t = 0.0f;
    active  = active && n_runs > 0 && n > 0;
    if (active) {
        const uint2 run = runs[0];
        t               = __uint_as_float(run.x);
        cnt             = run.y;
    }
    while (__any_sync(0xFFFFFFFFu, active)) {
        float tk = t;
        tk = G > 8u ? cone_steps(tk, g) : cone_steps_loop(tk, g);
        const float t_last = __shfl_sync(0xFFFFFFFFu, tk, group_lo + G - 1u);
        const uint32_t adv = active ? min(min(G, cnt - in_run), n - written) : 0u;
        if (g < adv) {
            const float3 p = ray_point(o, d_unit, tk);
            float* c       = stage + lane * 7u;
            c[0] = p.x, c[1] = p.y, c[2] = p.z, c[3] = kConeStep, c[4] = w3.x, c[5] = w3.y, c[6] = w3.z;
        }
        __syncwarp();
        if (active) {
            float* dst       = out + static_cast<uint64_t>(written) * 7u;
            const float* src = stage + group_lo * 7u;
            for (uint32_t q = g; q < 7u * adv; q += G) dst[q] = src[q];
            written += adv;
            in_run += adv;
            t = t_last + kConeStep;
            if (in_run == cnt) {
                ++r;
                in_run = 0;
                if (r == n_runs || written >= n) {
                    active = false;
                } else {
                    const uint2 run = runs[r];
                    t               = __uint_as_float(run.x);
                    cnt             = run.y;
                }
            }
        }
        __syncwarp();
    }
}

}  // namespace ngp
