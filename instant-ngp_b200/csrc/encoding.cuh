// Hash-grid encoding: per-level gather and trilinear interpolation shared by the encoding kernels
// (encoding.cu).  The arithmetic follows
// encode_grid_forward_kernel (ngp.train.cu:876-921) with fp32 accumulation: corner weights
// (wx * wy) * wz, fmaf over corners 0..7, one rounding to fp16 by the caller.
#pragma once

#include "common.cuh"

namespace ngp {

template <uint32_t F>
struct FeatureVec;
template <>
struct FeatureVec<1> {
    using type = __half;
};
template <>
struct FeatureVec<2> {
    using type = uint32_t;
};
template <>
struct FeatureVec<4> {
    using type = uint2;
};
template <>
struct FeatureVec<8> {
    using type = uint4;
};
template <>
struct FeatureVec<16> {
    using type = uint4;  // unused: pairs are formed for F <= 4 only
};

template <uint32_t F>
__device__ __forceinline__ void unpack(const typename FeatureVec<F>::type& v, float (&out)[F]) {
    if constexpr (F == 1) {
        out[0] = __half2float(v);
    } else {
        const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (uint32_t k = 0; k < F / 2; ++k) {
            const float2 f = __half22float2(h[k]);
            out[2 * k]     = f.x;
            out[2 * k + 1] = f.y;
        }
    }
}

// pos = fmaf(scale, x, 0.5); cell = floor(pos); frac = pos - cell (ngp.train.cu:188-193).
__device__ __forceinline__ void position_fraction(float x, float scale, float& frac, uint32_t& cell) {
    const float pos     = __fmaf_rn(scale, x, 0.5f);
    const float floored = floorf(pos);
    cell                = static_cast<uint32_t>(static_cast<int>(floored));
    frac                = __fsub_rn(pos, floored);
}

// Gather the 8 corners of `level` around point x (the level's cell and fraction in frac).
template <uint32_t F>
__device__ __forceinline__ void gather_level(const GridParams& grid, const typename FeatureVec<F>::type* __restrict__ tab, uint32_t level,
                                             const float (&x)[3], float (&frac)[3], typename FeatureVec<F>::type (&v)[8]) {
    const uint32_t off = grid.offsets[level], size = grid.offsets[level + 1] - off, res = grid.resolution[level];
    const float scale = grid.scale[level];
    uint32_t cell[3];
#pragma unroll
    for (uint32_t d = 0; d < 3; ++d) position_fraction(x[d], scale, frac[d], cell[d]);
    uint32_t idx[8];
    corner_indices((grid.dense_mask >> level) & 1u, size, res, cell[0], cell[1], cell[2], idx);
#pragma unroll
    for (uint32_t c = 0; c < 8; ++c) v[c] = __ldg(tab + off + idx[c]);
}

// Trilinear interpolation of the gathered corners: acc[f] = sum_c w_c * v_c[f] (fmaf, corner order).
template <uint32_t F>
__device__ __forceinline__ void interp_level(const float (&frac)[3], const typename FeatureVec<F>::type (&v)[8], float (&acc)[F]) {
#pragma unroll
    for (uint32_t f = 0; f < F; ++f) acc[f] = 0.0f;
#pragma unroll
    for (uint32_t corner = 0; corner < 8; ++corner) {
        const float wx = (corner & 1u) ? frac[0] : __fsub_rn(1.0f, frac[0]);
        const float wy = (corner & 2u) ? frac[1] : __fsub_rn(1.0f, frac[1]);
        const float wz = (corner & 4u) ? frac[2] : __fsub_rn(1.0f, frac[2]);
        const float w  = __fmul_rn(__fmul_rn(wx, wy), wz);
        float val[F];
        unpack<F>(v[corner], val);
#pragma unroll
        for (uint32_t f = 0; f < F; ++f) acc[f] = __fmaf_rn(w, val[f], acc[f]);
    }
}

}  // namespace ngp
