// Multiresolution hash-grid encoding, forward and backward, for sm_100a.
//
// Forward: point-major, one thread per point walking the levels two at a time (16 independent
// gathers in flight, the point read once); a corner's F features are one vector load (F=2:
// 32-bit half2) through the non-coherent read-only path.  The table (24 MB at the BASELINE
// configuration) is L2-resident on B200's 126 MB L2.  An optional row list selects the points.
// Backward: level-major, every CTA scatters one level for a chunk of points, the levels
// interleaved across consecutive CTAs; on coarse levels the lanes of a warp that share a cell sum
// their contributions first, and x-neighbour corners that pair up share one 16-byte atomic.
//
// Forward follows encode_grid_forward_kernel (ngp.train.cu:876-921) with fp32 accumulation
// (fmaf in corner order 0..7) instead of fp16 __hfma, rounded once to fp16.
// Backward follows encode_grid_backward_kernel (ngp.train.cu:923-960) but scatters into an
// fp32 gradient table with vector atomics (red.global.add.v2/v4.f32) instead of fp16 atomics.
#include "encoding.cuh"
#include "sampler.cuh"

// Tuning knob (compile-time; the default is the measured best on B200): levels up to this
// resolution pre-sum the lanes of a warp that share a cell before the backward's atomics.
#ifndef NGP_ENC_BWD_AGG_RES
#define NGP_ENC_BWD_AGG_RES 256
#endif

namespace ngp {
namespace {

constexpr uint32_t kEncodeThreads = 256u;

// Level and point-chunk of this CTA.  Interleaving the levels across consecutive CTAs spreads
// the atomic traffic of the small coarse tables over the whole kernel instead of issuing all of
// a coarse level's updates in the first wave.
__device__ __forceinline__ void cta_level_chunk(uint32_t n_levels, uint32_t& level, uint32_t& chunk) {
    level = blockIdx.x % n_levels;
    chunk = blockIdx.x / n_levels;
}

// Store N consecutive halves (N * 2 bytes, aligned to that size up to 16) with vector stores.
template <uint32_t N>
__device__ __forceinline__ void store_halves(__half* dst, const __half* v) {
    if constexpr (N * 2 >= 16) {
#pragma unroll
        for (uint32_t k = 0; k < N / 8; ++k) reinterpret_cast<uint4*>(dst)[k] = *reinterpret_cast<const uint4*>(v + 8 * k);
    } else if constexpr (N * 2 == 8) {
        *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(v);
    } else if constexpr (N * 2 == 4) {
        *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(v);
    } else {
        dst[0] = v[0];
    }
}

// Feature-major encoding of one point: levels LPI at a time, features to out[level * F + f][i].
template <uint32_t F, uint32_t LPI>
__device__ __forceinline__ void encode_point_features(const float (&x)[3], uint32_t i, const typename FeatureVec<F>::type* __restrict__ tab,
                                                      __half* __restrict__ out, uint32_t out_stride, const GridParams& grid) {
    for (uint32_t l0 = 0; l0 < grid.n_levels; l0 += LPI) {
        float frac[LPI][3];
        typename FeatureVec<F>::type v[LPI][8];
#pragma unroll
        for (uint32_t j = 0; j < LPI; ++j) gather_level<F>(grid, tab, min(l0 + j, grid.n_levels - 1u), x, frac[j], v[j]);
#pragma unroll
        for (uint32_t j = 0; j < LPI; ++j) {
            const uint32_t level = l0 + j;
            if (level >= grid.n_levels) break;
            float acc[F];
            interp_level<F>(frac[j], v[j], acc);
#pragma unroll
            for (uint32_t f = 0; f < F; ++f) out[static_cast<uint64_t>(level * F + f) * out_stride + i] = __float2half_rn(acc[f]);
        }
    }
}

// Point-major forward: a thread reads its point once and walks the levels LPI at a time (8 * LPI
// gathers in flight).  Same per-(point, level) arithmetic as encode_forward_kernel.
template <uint32_t F, uint32_t LPI, bool ROWS>
__global__ void __launch_bounds__(kEncodeThreads) encode_forward_points_kernel(const uint32_t n, const float* __restrict__ coords,
                                                                               const uint32_t coord_stride, const __half* __restrict__ table,
                                                                               __half* __restrict__ out, const uint32_t out_stride,
                                                                               const __grid_constant__ GridParams grid,
                                                                               const uint32_t* __restrict__ rows, const uint32_t* __restrict__ n_dev) {
    using Vec        = typename FeatureVec<F>::type;
    const uint32_t r    = blockIdx.x * kEncodeThreads + threadIdx.x;
    const bool live     = r < (n_dev != nullptr ? min(*n_dev, n) : n);
    if (!ROWS && !live) return;  // (row-major output: every lane takes part in the warp's write-out)
    // point i: row r itself, or the r-th entry of a row list (points read and written in place)
    const uint32_t i = live ? (rows != nullptr ? __ldg(rows + r) : r) : 0u;
    const float* c = coords + static_cast<uint64_t>(i) * coord_stride;
    const float x[3] = {live ? __ldg(c) : 0.0f, live ? __ldg(c + 1) : 0.0f, live ? __ldg(c + 2) : 0.0f};
    const Vec* tab   = reinterpret_cast<const Vec*>(table);
    __half pair_out[ROWS ? LPI * F : 1];
    // staging of row-major output rows (rows of 8, 16 or 32 halves), so that a warp writes whole
    // rows per store instruction
    constexpr uint32_t kStageHalves = 32;
    __shared__ __align__(16) __half stage[ROWS ? kEncodeThreads : 1][ROWS ? kStageHalves : 1];
    const uint32_t row_halves = grid.n_levels * F;
    const bool staged = ROWS && row_halves <= kStageHalves && row_halves % 8u == 0u && 32u % (row_halves / 8u) == 0u;
    if constexpr (!ROWS) {
        encode_point_features<F, LPI>(x, i, tab, out, out_stride, grid);
        return;
    }
    for (uint32_t l0 = 0; live && l0 < grid.n_levels; l0 += LPI) {
        float frac[LPI][3];
        Vec v[LPI][8];
#pragma unroll
        for (uint32_t j = 0; j < LPI; ++j) gather_level<F>(grid, tab, min(l0 + j, grid.n_levels - 1u), x, frac[j], v[j]);
#pragma unroll
        for (uint32_t j = 0; j < LPI; ++j) {
            const uint32_t level = l0 + j;
            if (level >= grid.n_levels) break;
            float acc[F];
            interp_level<F>(frac[j], v[j], acc);
            // this level's F features into the pair's vector, written once per level pair
#pragma unroll
            for (uint32_t f = 0; f < F; ++f) pair_out[j * F + f] = __float2half_rn(acc[f]);
        }
        // row-major [i][n_levels * F]: the level pair's LPI * F halves go to this thread's staged
        // row (written out coalesced below), or straight to the row when not staged
        __half* dst = staged ? &stage[threadIdx.x][l0 * F] : out + static_cast<uint64_t>(i) * (grid.n_levels * F) + l0 * F;
        if (l0 + LPI <= grid.n_levels) {
            store_halves<LPI * F>(dst, pair_out);
        } else {
            for (uint32_t k = 0; k < (grid.n_levels - l0) * F; ++k) dst[k] = pair_out[k];
        }
    }
    {
        if (staged) {
            // The warp's rows leave as 16-byte chunks: in round k, lane l writes chunk l % C of the
            // row of lane k * (32 / C) + l / C (C chunks per row), so each store instruction writes
            // 32 / C whole rows instead of one strided piece of every row.
            const uint32_t lane = threadIdx.x & 31u, wbase = threadIdx.x & ~31u;
            __syncwarp();  // the warp's staged rows are visible to every lane
            const uint32_t live_lanes = __ballot_sync(0xFFFFFFFFu, live);
            const uint32_t C = (grid.n_levels * F) / 8u, per = 32u / C;
            for (uint32_t k = 0; k < C; ++k) {
                const uint32_t src = k * per + lane / C, chunk = lane % C;
                const uint32_t row = __shfl_sync(0xFFFFFFFFu, i, src);
                if ((live_lanes >> src) & 1u)
                    reinterpret_cast<uint4*>(out + static_cast<uint64_t>(row) * (C * 8u))[chunk] =
                        *reinterpret_cast<const uint4*>(&stage[wbase + src][chunk * 8u]);
            }
        }
    }
}

// K2 + encoding of the warm-up grid samples (all 2^21 samples uniform, the first 256 steps):
// thread g makes the sample whose first cell is g (cell order, as
// generate_grid_samples_ordered_kernel: the same position and cell as K2's sample) and encodes
// it directly, writing its cell index; the position never goes to memory.
template <uint32_t F, uint32_t LPI>
__global__ void __launch_bounds__(kEncodeThreads) encode_grid_samples_kernel(uint32_t ema_step, uint64_t base_state, const float* __restrict__ values,
                                                                             uint32_t* __restrict__ indices, const __half* __restrict__ table,
                                                                             __half* __restrict__ out, const uint32_t out_stride,
                                                                             const __grid_constant__ GridParams grid) {
    __shared__ uint64_t jm[64], jp[64];
    if (threadIdx.x < 64) jm[threadIdx.x] = c_pcg_jump.mult[threadIdx.x];
    else if (threadIdx.x < 128) jp[threadIdx.x - 64] = c_pcg_jump.plus[threadIdx.x - 64];
    __syncthreads();
    const uint32_t g   = blockIdx.x * kEncodeThreads + threadIdx.x;  // cell (Morton index), < 2^21
    const uint32_t rel = (g - (kGridHashAdd & (kGridCells - 1u))) * kGridHashMulInv;
    const uint32_t i   = (rel - ema_step * kGridCells) & (kGridCells - 1u);
    float x[3];
    uint32_t idx;
    grid_sample_position(i, kGridCells, ema_step, -0.01f, base_state, jm, jp, values, x, idx);
    indices[g] = idx;
    encode_point_features<F, LPI>(x, g, reinterpret_cast<const typename FeatureVec<F>::type*>(table), out, out_stride, grid);
}

template <uint32_t F>
__device__ __forceinline__ void scatter_add(float* dst, const float (&g)[F]) {
    if constexpr (F == 1) {
        atomicAdd(dst, g[0]);
    } else if constexpr (F == 2) {
        atomicAdd(reinterpret_cast<float2*>(dst), make_float2(g[0], g[1]));
    } else if constexpr (F == 4) {
        atomicAdd(reinterpret_cast<float4*>(dst), make_float4(g[0], g[1], g[2], g[3]));
    } else {
        atomicAdd(reinterpret_cast<float4*>(dst), make_float4(g[0], g[1], g[2], g[3]));
        atomicAdd(reinterpret_cast<float4*>(dst + 4), make_float4(g[4], g[5], g[6], g[7]));
    }
}

// Scatter one (point, level) gradient: the 8 corner contributions (corner weights in the forward
// kernel's order, (wx * wy) * wz, times dy).
template <uint32_t F>
__device__ __forceinline__ void scatter_level(const float (&x)[3], const float (&g)[F], float* __restrict__ table_grad, const GridParams& grid,
                                              uint32_t level) {
    const uint32_t level_offset = grid.offsets[level];
    const uint32_t hashmap_size = grid.offsets[level + 1] - level_offset;
    const uint32_t resolution   = grid.resolution[level];
    const float scale           = grid.scale[level];
    float* __restrict__ lvl     = table_grad + static_cast<uint64_t>(level_offset) * F;
    float frac[3];
    uint32_t cell[3];
#pragma unroll
    for (uint32_t d = 0; d < 3; ++d) position_fraction(x[d], scale, frac[d], cell[d]);

    uint32_t idx[8];
    corner_indices((grid.dense_mask >> level) & 1u, hashmap_size, resolution, cell[0], cell[1], cell[2], idx);
    const float wx0 = __fsub_rn(1.0f, frac[0]), wx1 = frac[0];
#pragma unroll
    for (uint32_t yz = 0; yz < 4; ++yz) {
        const float wy     = (yz & 1u) ? frac[1] : __fsub_rn(1.0f, frac[1]);
        const float wz     = (yz & 2u) ? frac[2] : __fsub_rn(1.0f, frac[2]);
        const float w0     = __fmul_rn(__fmul_rn(wx0, wy), wz);
        const float w1     = __fmul_rn(__fmul_rn(wx1, wy), wz);
        const uint32_t i0  = idx[2 * yz], i1 = idx[2 * yz + 1];
        float c0[F], c1[F];
#pragma unroll
        for (uint32_t f = 0; f < F; ++f) {
            c0[f] = __fmul_rn(w0, g[f]);
            c1[f] = __fmul_rn(w1, g[f]);
        }
        if constexpr (F <= 2) {
            // Entries 2k and 2k+1 share one 16-byte (F=2) / 8-byte (F=1) aligned slot: one atomic.
            if ((i0 ^ i1) == 1u) {
                const uint32_t lo = i0 < i1 ? i0 : i1;
                float pair[2 * F];
#pragma unroll
                for (uint32_t f = 0; f < F; ++f) {
                    pair[f]     = i0 < i1 ? c0[f] : c1[f];
                    pair[F + f] = i0 < i1 ? c1[f] : c0[f];
                }
                scatter_add<2 * F>(lvl + static_cast<uint64_t>(lo) * F, pair);
                continue;
            }
        }
        scatter_add<F>(lvl + static_cast<uint64_t>(i0) * F, c0);
        scatter_add<F>(lvl + static_cast<uint64_t>(i1) * F, c1);
    }
}

template <uint32_t F>
__device__ __forceinline__ void load_dy(const __half* __restrict__ dy, uint32_t dy_stride, uint32_t level, uint32_t i, float (&g)[F]) {
#pragma unroll
    for (uint32_t f = 0; f < F; ++f) g[f] = __half2float(dy[static_cast<uint64_t>(level * F + f) * dy_stride + i]);
}

// Warp-aggregated scatter for coarse levels: consecutive points (samples along one ray) often
// fall into the same cell and so update the same 8 corners.  The lanes of a warp that share a
// cell add their 8 corner contributions in lane order, and only the lowest of them issues the
// atomics.  `stage` is this warp's [32][8 * F] shared-memory slot; `active` the lanes present.
template <uint32_t F>
__device__ __forceinline__ void scatter_level_warp(const float (&x)[3], const float (&g)[F], float* __restrict__ table_grad, const GridParams& grid,
                                                   uint32_t level, uint32_t active, float* __restrict__ stage) {
    const uint32_t level_offset = grid.offsets[level];
    const uint32_t hashmap_size = grid.offsets[level + 1] - level_offset;
    const uint32_t resolution   = grid.resolution[level];
    const float scale           = grid.scale[level];
    float* __restrict__ lvl     = table_grad + static_cast<uint64_t>(level_offset) * F;
    float frac[3];
    uint32_t cell[3];
#pragma unroll
    for (uint32_t d = 0; d < 3; ++d) position_fraction(x[d], scale, frac[d], cell[d]);
    const uint32_t lane  = threadIdx.x & 31u;
    const uint64_t key   = cell[0] | (static_cast<uint64_t>(cell[1]) << 21) | (static_cast<uint64_t>(cell[2]) << 42);
    const uint32_t peers = __match_any_sync(active, key);
    const bool lone      = __popc(peers) == 1;

    float c[8][F];
    const float wx0 = __fsub_rn(1.0f, frac[0]), wx1 = frac[0];
#pragma unroll
    for (uint32_t yz = 0; yz < 4; ++yz) {
        const float wy = (yz & 1u) ? frac[1] : __fsub_rn(1.0f, frac[1]);
        const float wz = (yz & 2u) ? frac[2] : __fsub_rn(1.0f, frac[2]);
        const float w0 = __fmul_rn(__fmul_rn(wx0, wy), wz);
        const float w1 = __fmul_rn(__fmul_rn(wx1, wy), wz);
#pragma unroll
        for (uint32_t f = 0; f < F; ++f) {
            c[2 * yz][f]     = __fmul_rn(w0, g[f]);
            c[2 * yz + 1][f] = __fmul_rn(w1, g[f]);
        }
    }
    if (!lone) {
        float* mine = stage + lane * (8u * F);
#pragma unroll
        for (uint32_t k = 0; k < 8; ++k)
#pragma unroll
            for (uint32_t f = 0; f < F; ++f) mine[k * F + f] = c[k][f];
    }
    __syncwarp(active);
    const bool leader = lone || (static_cast<uint32_t>(__ffs(peers)) - 1u) == lane;
    if (!lone && leader) {
        for (uint32_t rest = peers & (peers - 1u); rest; rest &= rest - 1u) {
            const float* other = stage + (static_cast<uint32_t>(__ffs(rest)) - 1u) * (8u * F);
#pragma unroll
            for (uint32_t k = 0; k < 8; ++k)
#pragma unroll
                for (uint32_t f = 0; f < F; ++f) c[k][f] += other[k * F + f];
        }
    }
    __syncwarp(active);
    if (!leader) return;
    uint32_t idx[8];
    corner_indices((grid.dense_mask >> level) & 1u, hashmap_size, resolution, cell[0], cell[1], cell[2], idx);
#pragma unroll
    for (uint32_t yz = 0; yz < 4; ++yz) {
        const uint32_t i0 = idx[2 * yz], i1 = idx[2 * yz + 1];
        if ((i0 ^ i1) == 1u) {
            const uint32_t lo = i0 < i1 ? i0 : i1;
            float pair[2 * F];
#pragma unroll
            for (uint32_t f = 0; f < F; ++f) {
                pair[f]     = i0 < i1 ? c[2 * yz][f] : c[2 * yz + 1][f];
                pair[F + f] = i0 < i1 ? c[2 * yz + 1][f] : c[2 * yz][f];
            }
            scatter_add<2 * F>(lvl + static_cast<uint64_t>(lo) * F, pair);
        } else {
            scatter_add<F>(lvl + static_cast<uint64_t>(i0) * F, c[2 * yz]);
            scatter_add<F>(lvl + static_cast<uint64_t>(i1) * F, c[2 * yz + 1]);
        }
    }
}

// Level-major backward: each CTA scatters one level for a chunk of points.
template <uint32_t F>
__global__ void __launch_bounds__(kEncodeThreads) encode_backward_kernel(const uint32_t n, const float* __restrict__ coords,
                                                                         const uint32_t coord_stride,
                                                                         const __half* __restrict__ dy, const uint32_t dy_stride,
                                                                         float* __restrict__ table_grad,
                                                                         const __grid_constant__ GridParams grid, const uint32_t* __restrict__ rows) {
    uint32_t level, chunk;
    cta_level_chunk(grid.n_levels, level, chunk);
    const uint32_t i = chunk * kEncodeThreads + threadIdx.x;
    if (i >= n) return;
    float g[F];
    load_dy<F>(dy, dy_stride, level, i, g);
    // point i's record: row i, or the sample rows[i] of a row list
    const float* c    = coords + static_cast<uint64_t>(rows != nullptr ? __ldg(rows + i) : i) * coord_stride;
    const float x[3]  = {__ldg(c), __ldg(c + 1), __ldg(c + 2)};
    if constexpr (F <= 2 && NGP_ENC_BWD_AGG_RES > 0) {
        if (grid.resolution[level] <= NGP_ENC_BWD_AGG_RES) {
            __shared__ float stage[kEncodeThreads / 32u][32u * 8u * F];
            scatter_level_warp<F>(x, g, table_grad, grid, level, __activemask(), stage[threadIdx.x >> 5]);
            return;
        }
    }
    scatter_level<F>(x, g, table_grad, grid, level);
}

int launch_points_forward(const ngp_grid_layout& layout, const GridParams& grid, uint32_t n, const float* coords, uint32_t coord_stride,
                          const uint16_t* table, uint16_t* out, uint32_t out_stride, const uint32_t* rows, const uint32_t* n_dev, cudaStream_t s) {
    constexpr uint32_t lpi = 2;  // levels in flight per thread (1 and 4 measured slower)
    const uint32_t blocks  = (n + kEncodeThreads - 1) / kEncodeThreads;
    const auto* t          = reinterpret_cast<const __half*>(table);
    auto* o                = reinterpret_cast<__half*>(out);
    const bool row_major   = rows_layout(out_stride);
#define NGP_ENC_FWD(FF)                                                                                                              \
    (row_major ? encode_forward_points_kernel<FF, lpi, true><<<blocks, kEncodeThreads, 0, s>>>(n, coords, coord_stride, t, o, out_stride, grid, rows, n_dev) \
               : encode_forward_points_kernel<FF, lpi, false><<<blocks, kEncodeThreads, 0, s>>>(n, coords, coord_stride, t, o, out_stride, grid, rows, n_dev))
    switch (layout.features_per_level) {
        case 1: NGP_ENC_FWD(1); break;
        case 2: NGP_ENC_FWD(2); break;
        case 4: NGP_ENC_FWD(4); break;
        default: NGP_ENC_FWD(8); break;
    }
#undef NGP_ENC_FWD
    return check_launch("encode_forward_points_kernel");
}

int validate_layout(const ngp_grid_layout* layout) {
    if (layout == nullptr) return fail(NGP_ERR_INVALID, "grid layout is null");
    if (layout->n_levels == 0 || layout->n_levels > NGP_MAX_LEVELS) return fail(NGP_ERR_INVALID, "grid layout: bad level count");
    const uint32_t F = layout->features_per_level;
    if (F != 1 && F != 2 && F != 4 && F != 8) return fail(NGP_ERR_INVALID, "grid layout: features per level must be 1, 2, 4 or 8");
    return NGP_OK;
}

}  // namespace

}  // namespace ngp

using namespace ngp;

extern "C" int ngp_encode_grid_forward(const ngp_grid_layout* layout, uint32_t n, const float* coords, uint32_t coord_stride,
                                       const uint16_t* table, uint16_t* out, uint32_t out_stride, void* stream) {
    clear_error();
    NGP_TRY(validate_layout(layout));
    if (n == 0) return NGP_OK;
    if (coords == nullptr || table == nullptr || out == nullptr) return fail(NGP_ERR_INVALID, "encode forward: null pointer");
    if (coord_stride < 3 || (!rows_layout(out_stride) && out_stride < n)) return fail(NGP_ERR_INVALID, "encode forward: bad stride");
    const GridParams grid = make_grid_params(*layout);
    return launch_points_forward(*layout, grid, n, coords, coord_stride, table, out, out_stride, nullptr, nullptr, as_stream(stream));
}

extern "C" int ngp_encode_grid_forward_rows(const ngp_grid_layout* layout, uint32_t max_rows, const uint32_t* rows, const uint32_t* n_rows,
                                            const float* coords, uint32_t coord_stride, const uint16_t* table, uint16_t* out, uint32_t out_stride,
                                            void* stream) {
    clear_error();
    NGP_TRY(validate_layout(layout));
    if (max_rows == 0) return NGP_OK;
    if (rows == nullptr || coords == nullptr || table == nullptr || out == nullptr) return fail(NGP_ERR_INVALID, "encode forward rows: null pointer");
    if (coord_stride < 3) return fail(NGP_ERR_INVALID, "encode forward rows: bad stride");
    return launch_points_forward(*layout, make_grid_params(*layout), max_rows, coords, coord_stride, table, out, out_stride, rows, n_rows,
                                 as_stream(stream));
}

namespace ngp {
namespace {
int encode_backward_launch(const ngp_grid_layout* layout, uint32_t n, const uint32_t* rows, const float* coords, uint32_t coord_stride,
                           const uint16_t* dy, uint32_t dy_stride, float* table_grad, void* stream) {
    NGP_TRY(validate_layout(layout));
    if (n == 0) return NGP_OK;
    if (coords == nullptr || dy == nullptr || table_grad == nullptr) return fail(NGP_ERR_INVALID, "encode backward: null pointer");
    if (coord_stride < 3 || dy_stride < n) return fail(NGP_ERR_INVALID, "encode backward: bad stride");
    const GridParams grid = make_grid_params(*layout);
    const auto* g = reinterpret_cast<const __half*>(dy);
    const dim3 blocks    = dim3(((n + kEncodeThreads - 1) / kEncodeThreads) * layout->n_levels);
    const cudaStream_t s = as_stream(stream);
    switch (layout->features_per_level) {
        case 1: encode_backward_kernel<1><<<blocks, kEncodeThreads, 0, s>>>(n, coords, coord_stride, g, dy_stride, table_grad, grid, rows); break;
        case 2: encode_backward_kernel<2><<<blocks, kEncodeThreads, 0, s>>>(n, coords, coord_stride, g, dy_stride, table_grad, grid, rows); break;
        case 4: encode_backward_kernel<4><<<blocks, kEncodeThreads, 0, s>>>(n, coords, coord_stride, g, dy_stride, table_grad, grid, rows); break;
        default: encode_backward_kernel<8><<<blocks, kEncodeThreads, 0, s>>>(n, coords, coord_stride, g, dy_stride, table_grad, grid, rows); break;
    }
    return check_launch("encode_backward_kernel");
}
}  // namespace
}  // namespace ngp

extern "C" int ngp_encode_grid_backward(const ngp_grid_layout* layout, uint32_t n, const float* coords, uint32_t coord_stride,
                                        const uint16_t* dy, uint32_t dy_stride, float* table_grad, void* stream) {
    clear_error();
    return encode_backward_launch(layout, n, nullptr, coords, coord_stride, dy, dy_stride, table_grad, stream);
}

extern "C" int ngp_encode_grid_backward_rows(const ngp_grid_layout* layout, uint32_t n, const uint32_t* rows, const float* coords,
                                             uint32_t coord_stride, const uint16_t* dy, uint32_t dy_stride, float* table_grad, void* stream) {
    clear_error();
    if (rows == nullptr) return fail(NGP_ERR_INVALID, "encode backward rows: null row list");
    return encode_backward_launch(layout, n, rows, coords, coord_stride, dy, dy_stride, table_grad, stream);
}

extern "C" int ngp_density_grid_encode_samples(const ngp_grid_layout* layout, uint32_t ema_step, const float* values, const uint16_t* table,
                                               uint16_t* out, uint32_t out_stride, uint32_t* indices, void* stream) {
    clear_error();
    NGP_TRY(validate_layout(layout));
    if (values == nullptr || table == nullptr || out == nullptr || indices == nullptr) return fail(NGP_ERR_INVALID, "grid encode samples: null pointer");
    if (out_stride < kGridCells) return fail(NGP_ERR_INVALID, "grid encode samples: bad stride");
    const GridParams grid = make_grid_params(*layout);
    // the set's stream before the per-sample jump: PCG32(1337) advanced by (2 ema_step + 1) << 32
    Pcg32 u{kTrainSeed};
    u.advance((static_cast<uint64_t>(ema_step) * 2ull + 1ull) << 32u);
    const auto* t      = reinterpret_cast<const __half*>(table);
    auto* o            = reinterpret_cast<__half*>(out);
    const uint32_t blk = kGridCells / kEncodeThreads;
    const cudaStream_t s = as_stream(stream);
    switch (layout->features_per_level) {
        case 1: encode_grid_samples_kernel<1, 2><<<blk, kEncodeThreads, 0, s>>>(ema_step, u.state, values, indices, t, o, out_stride, grid); break;
        case 2: encode_grid_samples_kernel<2, 2><<<blk, kEncodeThreads, 0, s>>>(ema_step, u.state, values, indices, t, o, out_stride, grid); break;
        case 4: encode_grid_samples_kernel<4, 2><<<blk, kEncodeThreads, 0, s>>>(ema_step, u.state, values, indices, t, o, out_stride, grid); break;
        default: encode_grid_samples_kernel<8, 2><<<blk, kEncodeThreads, 0, s>>>(ema_step, u.state, values, indices, t, o, out_stride, grid); break;
    }
    return check_launch("encode_grid_samples_kernel");
}
