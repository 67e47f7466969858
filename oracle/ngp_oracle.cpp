// ngp_oracle.cpp -- CPU restatement of the reference's NeRF hot path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library: only tests/,
// __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may load it.  The
// product path (instant-ngp_b200/) never links, loads or calls it.
//
// Every function restates, in scalar C++, the algorithm of the reference file:line it cites
// (Xayah-Graphics/instant-ngp, ngp.train.cu / ngp.train.h).  Parity pin: the reference has no
// tests or golden vectors of its own, so this oracle is pinned against outputs of the
// reference's own kernels, compiled from its sources into oracle/_ref/ and run on a B200;
// those outputs are committed as fixtures under tests/golden/ (see make_golden.py there).
//
// Floating point follows IEEE binary32 with no contraction (built with -ffp-contract=off);
// fused multiply-adds appear only where they are explicit (fmaf), as in the CUDA code.
// fp16 is the compiler's _Float16 (IEEE binary16, round-to-nearest-even conversions).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <thread>
#include <vector>

namespace {

using half = _Float16;

inline float h2f(uint16_t bits) {
    half h;
    std::memcpy(&h, &bits, 2);
    return static_cast<float>(h);
}
inline uint16_t f2h(float f) {
    const half h = static_cast<half>(f);
    uint16_t bits;
    std::memcpy(&bits, &h, 2);
    return bits;
}

// fp16 fused multiply-add with one rounding, as __hfma: the product of two binary16 values is
// exact in binary64 and so is its sum with a binary16 addend for every case that can change the
// binary16 result, so a binary64 fma followed by one conversion rounds like the hardware.
inline uint16_t hfma(uint16_t a, uint16_t b, uint16_t c) {
    const double r = std::fma(static_cast<double>(h2f(a)), static_cast<double>(h2f(b)), static_cast<double>(h2f(c)));
    const half h   = static_cast<half>(r);
    uint16_t bits;
    std::memcpy(&bits, &h, 2);
    return bits;
}

template <typename Fn>
void parallel_for(uint32_t n, int threads, Fn&& fn, uint32_t min_items = 1024) {
    if (threads <= 1 || n < min_items) {
        fn(0u, n);
        return;
    }
    std::vector<std::thread> pool;
    const uint32_t chunk = (n + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        const uint32_t b = std::min<uint32_t>(n, t * chunk), e = std::min<uint32_t>(n, b + chunk);
        if (b < e) pool.emplace_back([&, b, e] { fn(b, e); });
    }
    for (auto& th : pool) th.join();
}

// ---- PCG32 (ngp.train.cu:85-143) -----------------------------------------------------------
struct Pcg {
    uint64_t state, inc;
    explicit Pcg(uint64_t initstate, uint64_t initseq = 1u) {
        state = 0u;
        inc   = (initseq << 1u) | 1u;
        next();
        state += initstate;
        next();
    }
    uint32_t next() {
        const uint64_t old = state;
        state              = old * 0x5851f42d4c957f2dULL + inc;
        const uint32_t xs  = static_cast<uint32_t>(((old >> 18u) ^ old) >> 27u);
        const uint32_t rot = static_cast<uint32_t>(old >> 59u);
        return (xs >> rot) | (xs << ((~rot + 1u) & 31u));
    }
    float next_float() {
        const uint32_t bits = (next() >> 9u) | 0x3f800000u;
        float v;
        std::memcpy(&v, &bits, 4);
        return v - 1.0f;
    }
    void advance(uint64_t delta) {
        uint64_t cm = 0x5851f42d4c957f2dULL, cp = inc, am = 1u, ap = 0u;
        for (; delta > 0u; delta >>= 1u) {
            if (delta & 1u) {
                am *= cm;
                ap = ap * cm + cp;
            }
            cp = (cm + 1u) * cp;
            cm *= cm;
        }
        state = am * state + ap;
    }
};

// ---- grid index (ngp.train.cu:165-193) -----------------------------------------------------
inline uint32_t grid_index(uint32_t hashmap_size, uint32_t res, uint32_t x, uint32_t y, uint32_t z) {
    uint32_t stride = 1u, index = 0u;
    if (res <= 0x659u) {
        index += x * stride;
        stride *= res;
        index += y * stride;
        stride *= res;
        index += z * stride;
        stride *= res;
    } else {
        stride = 0xFFFFFFFFu;
    }
    if (hashmap_size < stride) index = x ^ (y * 2654435761u) ^ (z * 805459861u);
    return index % hashmap_size;
}

inline void pos_frac(float x, float scale, float& frac, uint32_t& cell) {
    const float pos = std::fmaf(scale, x, 0.5f);
    const float fl  = std::floor(pos);
    cell            = static_cast<uint32_t>(static_cast<int>(fl));
    frac            = pos - fl;
}

struct Layout {
    uint32_t L, F;
    const uint32_t* offsets;     // L + 1
    const uint32_t* resolution;  // L
    const float* scale;          // L
};

inline float corner_weight(uint32_t corner, const float frac[3]) {
    const float wx = (corner & 1u) ? frac[0] : 1.0f - frac[0];
    const float wy = (corner & 2u) ? frac[1] : 1.0f - frac[1];
    const float wz = (corner & 4u) ? frac[2] : 1.0f - frac[2];
    return (wx * wy) * wz;
}

inline uint32_t corner_index(const Layout& g, uint32_t l, uint32_t corner, const uint32_t cell[3]) {
    const uint32_t hs = g.offsets[l + 1] - g.offsets[l];
    return grid_index(hs, g.resolution[l], cell[0] + (corner & 1u), cell[1] + ((corner >> 1) & 1u), cell[2] + ((corner >> 2) & 1u));
}

}  // namespace

extern "C" {

// ---- layout (ngp.train.h:44-56; generalised scale of example.py:400-401) -------------------
int oracle_grid_layout(uint32_t L, uint32_t F, uint32_t log2T, uint32_t base, double log2_scale, uint32_t* offsets, uint32_t* resolution,
                       float* scale) {
    const uint64_t T = uint64_t{1} << log2T;
    uint64_t cursor  = 0;
    for (uint32_t l = 0; l < L; ++l) {
        const double s   = std::exp2(static_cast<double>(l) * log2_scale) * static_cast<double>(base) - 1.0;
        const uint64_t r = static_cast<uint64_t>(std::ceil(s)) + 1u;
        uint64_t p       = std::min<uint64_t>(r * r * r, std::numeric_limits<uint32_t>::max() / 2ull);
        p                = std::min<uint64_t>((p + 7u) / 8u * 8u, T);
        offsets[l]       = static_cast<uint32_t>(cursor);
        resolution[l]    = static_cast<uint32_t>(r);
        scale[l]         = static_cast<float>(s);
        cursor += p;
    }
    offsets[L] = static_cast<uint32_t>(cursor);
    (void)F;
    return 0;
}

uint32_t oracle_grid_index(uint32_t hashmap_size, uint32_t res, uint32_t x, uint32_t y, uint32_t z) { return grid_index(hashmap_size, res, x, y, z); }

// ---- encoding forward (ngp.train.cu:876-921) -----------------------------------------------
// mode 0: fp32 accumulation with fmaf in corner order (the CUDA library's arithmetic).
// mode 1: the reference's arithmetic -- weight rounded to fp16, fp16 __hfma accumulation.
void oracle_encode_forward(uint32_t L, uint32_t F, const uint32_t* offsets, const uint32_t* resolution, const float* scale, uint32_t n,
                           const float* coords, uint32_t coord_stride, const uint16_t* table, uint16_t* out, uint32_t out_stride, int mode,
                           int threads) {
    const Layout g{L, F, offsets, resolution, scale};
    parallel_for(n, threads, [&](uint32_t b, uint32_t e) {
        for (uint32_t i = b; i < e; ++i) {
            const float* c = coords + static_cast<uint64_t>(i) * coord_stride;
            for (uint32_t l = 0; l < L; ++l) {
                float frac[3];
                uint32_t cell[3];
                for (int d = 0; d < 3; ++d) pos_frac(c[d], scale[l], frac[d], cell[d]);
                const uint16_t* lvl = table + static_cast<uint64_t>(offsets[l]) * F;
                float acc[8]        = {};
                uint16_t hacc[8]    = {};
                for (uint32_t corner = 0; corner < 8; ++corner) {
                    const float w      = corner_weight(corner, frac);
                    const uint32_t idx = corner_index(g, l, corner, cell);
                    for (uint32_t f = 0; f < F; ++f) {
                        const uint16_t v = lvl[static_cast<uint64_t>(idx) * F + f];
                        if (mode == 0)
                            acc[f] = std::fmaf(w, h2f(v), acc[f]);
                        else
                            hacc[f] = hfma(f2h(w), v, hacc[f]);
                    }
                }
                for (uint32_t f = 0; f < F; ++f) out[static_cast<uint64_t>(l * F + f) * out_stride + i] = mode == 0 ? f2h(acc[f]) : hacc[f];
            }
        }
    });
}

// ---- encoding backward (ngp.train.cu:923-960) ----------------------------------------------
// grad[e*F+f] (fp64) += w * dy: exact-as-possible reference sums for tolerance checks.
// Threads split by level: levels own disjoint table ranges, so no two threads share an entry.
void oracle_encode_backward(uint32_t L, uint32_t F, const uint32_t* offsets, const uint32_t* resolution, const float* scale, uint32_t n,
                            const float* coords, uint32_t coord_stride, const uint16_t* dy, uint32_t dy_stride, double* grad, int threads) {
    const Layout g{L, F, offsets, resolution, scale};
    parallel_for(L, std::min<int>(threads, static_cast<int>(L)), [&](uint32_t lb, uint32_t le) {
        for (uint32_t l = lb; l < le; ++l) {
            double* lvl = grad + static_cast<uint64_t>(offsets[l]) * F;
            for (uint32_t i = 0; i < n; ++i) {
                const float* c = coords + static_cast<uint64_t>(i) * coord_stride;
                float frac[3];
                uint32_t cell[3];
                for (int d = 0; d < 3; ++d) pos_frac(c[d], scale[l], frac[d], cell[d]);
                for (uint32_t corner = 0; corner < 8; ++corner) {
                    const float w      = corner_weight(corner, frac);
                    const uint32_t idx = corner_index(g, l, corner, cell);
                    for (uint32_t f = 0; f < F; ++f)
                        lvl[static_cast<uint64_t>(idx) * F + f] += static_cast<double>(w) * static_cast<double>(h2f(dy[static_cast<uint64_t>(l * F + f) * dy_stride + i]));
                }
            }
        }
    }, 1u);
}

// ---- PCG32 stream (for pinning the device generator) ---------------------------------------
void oracle_pcg32(uint64_t initstate, uint64_t initseq, uint64_t advance, uint32_t count, uint32_t* out_uint, float* out_float) {
    Pcg a(initstate, initseq);
    a.advance(advance);
    Pcg b = a;
    for (uint32_t i = 0; i < count; ++i) {
        out_uint[i]  = a.next();
        out_float[i] = b.next_float();
    }
}

}  // extern "C"

// ======================================================================================
// Spherical harmonics (ngp.train.cu:962-993) and the fully fused MLPs (ngp.train.cu:1019-1236,
// 1660-1903).  Packed fp16 weights [out][in] at the reference offsets (ngp.train.h:58-78):
//   density W_in 64x32 @0, density W_out 16x64 @2048, rgb W_in 64x32 @3072,
//   rgb W_h 64x64 @5120, rgb W_out 16x64 @9216  (10,240 weights, no biases).
// Arithmetic restated with fp32 accumulation and one fp16 rounding per layer output, which is
// the CUDA library's arithmetic; the reference accumulates in fp16 (checked with tolerances).
// ======================================================================================
namespace {

constexpr uint32_t kWdIn = 0, kWdOut = 2048, kWrIn = 3072, kWrH = 5120, kWrOut = 9216, kMlpParams = 10240;

inline float rh(float v) { return h2f(f2h(v)); }  // round to fp16 and back

// Degree-4 real spherical harmonics of dir = 2 * warped - 1.  The products and sums are written
// out one IEEE operation at a time; the a*b+c forms use a single fused multiply-add.
void sh16(float wx, float wy, float wz, float out[16]) {
    const float x = wx * 2.0f - 1.0f, y = wy * 2.0f - 1.0f, z = wz * 2.0f - 1.0f;
    const float xy = x * y, xz = x * z, yz = y * z, x2 = x * x, y2 = y * y, z2 = z * z;
    out[0]  = 0.28209479177387814f;
    out[1]  = -0.48860251190291987f * y;
    out[2]  = 0.48860251190291987f * z;
    out[3]  = -0.48860251190291987f * x;
    out[4]  = 1.0925484305920792f * xy;
    out[5]  = -1.0925484305920792f * yz;
    out[6]  = std::fmaf(0.94617469575755997f, z2, -0.31539156525251999f);
    out[7]  = -1.0925484305920792f * xz;
    out[8]  = std::fmaf(0.54627421529603959f, x2, -(0.54627421529603959f * y2));
    out[9]  = (0.59004358992664352f * y) * std::fmaf(-3.0f, x2, y2);
    out[10] = (2.8906114426405538f * xy) * z;
    out[11] = (0.45704579946446572f * y) * std::fmaf(-5.0f, z2, 1.0f);
    out[12] = (0.3731763325901154f * z) * std::fmaf(5.0f, z2, -3.0f);
    out[13] = (0.45704579946446572f * x) * std::fmaf(-5.0f, z2, 1.0f);
    out[14] = (1.4453057213202769f * z) * (x2 - y2);
    out[15] = (0.59004358992664352f * x) * std::fmaf(3.0f, y2, -x2);
}

// y[o] = sum_k W[o][k] x[k] with an fp32 fmaf chain in k order.
template <int OUT, int IN>
void layer(const uint16_t* W, const float* x, float* y) {
    for (int o = 0; o < OUT; ++o) {
        float acc = 0.0f;
        for (int k = 0; k < IN; ++k) acc = std::fmaf(h2f(W[o * IN + k]), x[k], acc);
        y[o] = acc;
    }
}

struct RowActs {
    float x[32], hd[64], dout[16], ri[32], h1[64], h2[64], out[16];
};

void mlp_row_forward(const uint16_t* P, const float x16[32], const float dir[3], RowActs& a) {
    for (int k = 0; k < 32; ++k) a.x[k] = x16[k];
    float t[64];
    layer<64, 32>(P + kWdIn, a.x, t);
    for (int j = 0; j < 64; ++j) a.hd[j] = rh(std::max(t[j], 0.0f));
    layer<16, 64>(P + kWdOut, a.hd, t);
    for (int o = 0; o < 16; ++o) a.dout[o] = rh(t[o]);
    float sh[16];
    sh16(dir[0], dir[1], dir[2], sh);
    for (int k = 0; k < 16; ++k) {
        a.ri[k]      = a.dout[k];
        a.ri[16 + k] = rh(sh[k]);
    }
    layer<64, 32>(P + kWrIn, a.ri, t);
    for (int j = 0; j < 64; ++j) a.h1[j] = rh(std::max(t[j], 0.0f));
    layer<64, 64>(P + kWrH, a.h1, t);
    for (int j = 0; j < 64; ++j) a.h2[j] = rh(std::max(t[j], 0.0f));
    layer<16, 64>(P + kWrOut, a.h2, t);
    for (int o = 0; o < 16; ++o) a.out[o] = rh(t[o]);
    a.out[3] = a.dout[0];
}

}  // namespace

extern "C" {

// SH encoding of n sample records (dirs at floats 4..6 of each 7-float record) -> fp16 [16][n].
void oracle_sh_encode(uint32_t n, const float* coords, uint32_t coord_stride, uint16_t* out) {
    for (uint32_t i = 0; i < n; ++i) {
        const float* c = coords + static_cast<uint64_t>(i) * coord_stride;
        float sh[16];
        sh16(c[4], c[5], c[6], sh);
        for (int k = 0; k < 16; ++k) out[static_cast<uint64_t>(k) * n + i] = f2h(sh[k]);
    }
}

// Network forward (evaluate_network, ngp.train.cu:1494-1524): x fp16 feature-major [32][x_stride],
// sample records for the view directions -> out fp16 [n][16] (ch 0-2 rgb raw, ch 3 density raw).
void oracle_mlp_forward(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const float* coords, uint32_t coord_stride,
                        uint16_t* out, int threads) {
    parallel_for(n, threads, [&](uint32_t b, uint32_t e) {
        for (uint32_t i = b; i < e; ++i) {
            float xr[32];
            for (int k = 0; k < 32; ++k) xr[k] = h2f(x[static_cast<uint64_t>(k) * x_stride + i]);
            const float* c = coords + static_cast<uint64_t>(i) * coord_stride;
            RowActs a;
            mlp_row_forward(params, xr, c + 4, a);
            for (int o = 0; o < 16; ++o) out[static_cast<uint64_t>(i) * 16 + o] = f2h(a.out[o]);
        }
    });
}

// Density network only (update_density_grid, ngp.train.cu:1569-1573): raw density (ch 0) -> out[n].
void oracle_density_forward(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, uint16_t* out) {
    for (uint32_t i = 0; i < n; ++i) {
        float xr[32], t[64], hd[64], d[16];
        for (int k = 0; k < 32; ++k) xr[k] = h2f(x[static_cast<uint64_t>(k) * x_stride + i]);
        layer<64, 32>(params + kWdIn, xr, t);
        for (int j = 0; j < 64; ++j) hd[j] = rh(std::max(t[j], 0.0f));
        layer<16, 64>(params + kWdOut, hd, d);
        out[i] = f2h(d[0]);
    }
}

// Network backward (backward_network, ngp.train.cu:1686-1903) for n rows:
// dy fp16 [n][16] (ch 0-2 rgb, ch 3 density; others ignored as extract_rgb_gradients does)
// -> dx fp16 [32][dx_stride] (gradient w.r.t. the encoded input) and dW fp64 [10240] (summed).
}  // extern "C"

namespace {
// Rows [begin, end) of the network backward; dW accumulates in row order.
void mlp_backward_rows(uint32_t begin, uint32_t end, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const float* coords,
                       uint32_t coord_stride, const uint16_t* dy, uint16_t* dx, uint32_t dx_stride, double* dW) {
    const uint16_t* P = params;
    for (uint32_t i = begin; i < end; ++i) {
        float xr[32];
        for (int k = 0; k < 32; ++k) xr[k] = h2f(x[static_cast<uint64_t>(k) * x_stride + i]);
        RowActs a;
        mlp_row_forward(P, xr, coords + static_cast<uint64_t>(i) * coord_stride + 4, a);
        float g[16] = {};
        for (int o = 0; o < 3; ++o) g[o] = h2f(dy[static_cast<uint64_t>(i) * 16 + o]);
        const float gd = h2f(dy[static_cast<uint64_t>(i) * 16 + 3]);
        float dh2[64], dh1[64], dxr[32], ddo[16], dhd[64];
        for (int j = 0; j < 64; ++j) {
            float acc = 0.0f;
            for (int o = 0; o < 16; ++o) acc = std::fmaf(g[o], h2f(P[kWrOut + o * 64 + j]), acc);
            dh2[j] = a.h2[j] > 0.0f ? rh(acc) : 0.0f;
        }
        for (int k = 0; k < 64; ++k) {
            float acc = 0.0f;
            for (int j = 0; j < 64; ++j) acc = std::fmaf(dh2[j], h2f(P[kWrH + j * 64 + k]), acc);
            dh1[k] = a.h1[k] > 0.0f ? rh(acc) : 0.0f;
        }
        for (int k = 0; k < 32; ++k) {
            float acc = 0.0f;
            for (int j = 0; j < 64; ++j) acc = std::fmaf(dh1[j], h2f(P[kWrIn + j * 32 + k]), acc);
            dxr[k] = acc;
        }
        for (int o = 0; o < 16; ++o) ddo[o] = rh(o == 0 ? dxr[0] + gd : dxr[o]);
        for (int j = 0; j < 64; ++j) {
            float acc = 0.0f;
            for (int o = 0; o < 16; ++o) acc = std::fmaf(ddo[o], h2f(P[kWdOut + o * 64 + j]), acc);
            dhd[j] = a.hd[j] > 0.0f ? rh(acc) : 0.0f;
        }
        for (int k = 0; k < 32; ++k) {
            float acc = 0.0f;
            for (int j = 0; j < 64; ++j) acc = std::fmaf(dhd[j], h2f(P[kWdIn + j * 32 + k]), acc);
            dx[static_cast<uint64_t>(k) * dx_stride + i] = f2h(acc);
        }
        for (int o = 0; o < 16; ++o)
            for (int j = 0; j < 64; ++j) dW[kWrOut + o * 64 + j] += static_cast<double>(g[o]) * a.h2[j];
        for (int j = 0; j < 64; ++j)
            for (int k = 0; k < 64; ++k) dW[kWrH + j * 64 + k] += static_cast<double>(dh2[j]) * a.h1[k];
        for (int j = 0; j < 64; ++j)
            for (int k = 0; k < 32; ++k) dW[kWrIn + j * 32 + k] += static_cast<double>(dh1[j]) * a.ri[k];
        for (int o = 0; o < 16; ++o)
            for (int j = 0; j < 64; ++j) dW[kWdOut + o * 64 + j] += static_cast<double>(ddo[o]) * a.hd[j];
        for (int j = 0; j < 64; ++j)
            for (int k = 0; k < 32; ++k) dW[kWdIn + j * 32 + k] += static_cast<double>(dhd[j]) * a.x[k];
    }
}
}  // namespace

extern "C" {

void oracle_mlp_backward(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const float* coords, uint32_t coord_stride,
                         const uint16_t* dy, uint16_t* dx, uint32_t dx_stride, double* dW) {
    mlp_backward_rows(0, n, params, x, x_stride, coords, coord_stride, dy, dx, dx_stride, dW);
}

// The same over `threads` host threads (CPU baseline timing): each thread sums its rows' weight
// gradients, the partial sums are added in thread order.
void oracle_mlp_backward_mt(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const float* coords, uint32_t coord_stride,
                            const uint16_t* dy, uint16_t* dx, uint32_t dx_stride, double* dW, int threads) {
    const int t_count = std::max(1, threads);
    std::vector<std::vector<double>> partial(static_cast<size_t>(t_count), std::vector<double>(10240, 0.0));
    std::vector<std::thread> pool;
    const uint32_t chunk = (n + t_count - 1) / t_count;
    for (int t = 0; t < t_count; ++t) {
        const uint32_t b = std::min(n, t * chunk), e = std::min(n, b + chunk);
        pool.emplace_back([&, t, b, e] { mlp_backward_rows(b, e, params, x, x_stride, coords, coord_stride, dy, dx, dx_stride, partial[t].data()); });
    }
    for (auto& th : pool) th.join();
    for (int t = 0; t < t_count; ++t)
        for (int k = 0; k < 10240; ++k) dW[k] += partial[t][k];
}

}  // extern "C"

// ======================================================================================
// Occupancy grid and ray marching (ngp.train.cu:195-249, 383-474, 476-578, 580-667).
// The a*b+c forms that the reference's compiler contracts are written as std::fmaf, as in the
// CUDA library, so counts and positions can be compared bit for bit.
// ======================================================================================
namespace {

constexpr float kDt = 1.73205080757f / 1024.0f;

inline uint32_t spread3(uint32_t v) {
    v = (v * 0x00010001u) & 0xFF0000FFu;
    v = (v * 0x00000101u) & 0x0F00F00Fu;
    v = (v * 0x00000011u) & 0xC30C30C3u;
    v = (v * 0x00000005u) & 0x49249249u;
    return v;
}
inline uint32_t compact3(uint32_t v) {
    v &= 0x49249249u;
    v = (v | (v >> 2u)) & 0xC30C30C3u;
    v = (v | (v >> 4u)) & 0x0F00F00Fu;
    v = (v | (v >> 8u)) & 0xFF0000FFu;
    v = (v | (v >> 16u)) & 0x0000FFFFu;
    return v;
}

struct V3 {
    float x, y, z;
};

inline bool inside(V3 p) { return p.x >= 0.0f && p.x <= 1.0f && p.y >= 0.0f && p.y <= 1.0f && p.z >= 0.0f && p.z <= 1.0f; }

inline bool hit_cube(V3 o, V3 d, float& tmin_out) {
    const V3 inv = {1.0f / d.x, 1.0f / d.y, 1.0f / d.z};
    const V3 t0  = {-o.x * inv.x, -o.y * inv.y, -o.z * inv.z};
    const V3 t1  = {(1.0f - o.x) * inv.x, (1.0f - o.y) * inv.y, (1.0f - o.z) * inv.z};
    const float tmin = std::fmax(std::fmax(std::fmin(t0.x, t1.x), std::fmin(t0.y, t1.y)), std::fmin(t0.z, t1.z));
    const float tmax = std::fmin(std::fmin(std::fmax(t0.x, t1.x), std::fmax(t0.y, t1.y)), std::fmax(t0.z, t1.z));
    tmin_out         = std::fmax(tmin, 0.0f);
    return tmax >= tmin_out;
}

inline bool occ(V3 p, const uint8_t* bits) {
    const int x = static_cast<int>(p.x * 128.0f), y = static_cast<int>(p.y * 128.0f), z = static_cast<int>(p.z * 128.0f);
    if (x < 0 || x >= 128 || y < 0 || y >= 128 || z < 0 || z >= 128) return false;
    const uint32_t idx = spread3(x) | (spread3(y) << 1) | (spread3(z) << 2);
    return (bits[idx / 8] >> (idx % 8)) & 1u;
}

inline float skip_voxel(float t, V3 pos, V3 d, V3 inv) {
    const V3 p     = {(pos.x - 0.5f) * 128.0f, (pos.y - 0.5f) * 128.0f, (pos.z - 0.5f) * 128.0f};
    const float tx = (std::floor(std::fmaf(0.5f, std::copysign(1.0f, d.x), p.x + 0.5f)) - p.x) * inv.x;
    const float ty = (std::floor(std::fmaf(0.5f, std::copysign(1.0f, d.y), p.y + 0.5f)) - p.y) * inv.y;
    const float tz = (std::floor(std::fmaf(0.5f, std::copysign(1.0f, d.z), p.z + 0.5f)) - p.z) * inv.z;
    const float tt = t + std::fmax(std::fmin(std::fmin(tx, ty), tz) / 128.0f, 0.0f);
    return std::fmaf(std::ceil(std::fmax((tt - t) / kDt, 0.5f)), kDt, t);
}

inline V3 at(V3 o, V3 d, float t) { return {std::fmaf(d.x, t, o.x), std::fmaf(d.y, t, o.y), std::fmaf(d.z, t, o.z)}; }

// March one ray; write up to `limit` records into out (may be null to count only).  t_last
// (optional) receives the t of the last sample.
uint32_t march(V3 o, V3 d, float start, const uint8_t* bits, float* out, uint32_t limit, float* t_last = nullptr) {
    const V3 inv  = {1.0f / d.x, 1.0f / d.y, 1.0f / d.z};
    const V3 warp = {(d.x + 1.0f) * 0.5f, (d.y + 1.0f) * 0.5f, (d.z + 1.0f) * 0.5f};
    uint32_t n    = 0;
    float t       = start;
    while (n < limit) {
        const V3 p = at(o, d, t);
        if (!inside(p)) break;
        if (occ(p, bits)) {
            if (out != nullptr) {
                float* c = out + static_cast<uint64_t>(n) * 7u;
                c[0] = p.x, c[1] = p.y, c[2] = p.z, c[3] = kDt, c[4] = warp.x, c[5] = warp.y, c[6] = warp.z;
            }
            ++n;
            if (t_last != nullptr) *t_last = t;
            t += kDt;
        } else {
            t = skip_voxel(t, p, d, inv);
        }
    }
    return n;
}

}  // namespace

extern "C" {

// Explicit rays [n][6] (origin, unit dir); start = tmin + U*dt with U the third draw of the
// training PCG32 stream of ray i at `step` (jitter) or tmin + dt/2.  Samples in ray order.
// Returns the total number of samples before the limit.
uint32_t oracle_march_rays(uint32_t n, const float* rays, int jitter, uint32_t step, const uint8_t* bits, uint32_t sample_limit, uint32_t* numsteps,
                           float* coords) {
    uint32_t base = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const float* q = rays + static_cast<uint64_t>(i) * 6u;
        const V3 o = {q[0], q[1], q[2]}, d = {q[3], q[4], q[5]};
        float tmin      = 0.0f;
        uint32_t steps  = 0;
        float start     = 0.0f;
        if (hit_cube(o, d, tmin)) {
            if (jitter) {
                Pcg rng(1337u);
                rng.advance(static_cast<uint64_t>(step) << 32u);
                rng.advance(static_cast<uint64_t>(i) * 16u);
                rng.next_float();
                rng.next_float();
                start = std::fmaf(rng.next_float(), kDt, tmin);
            } else {
                start = tmin + 0.5f * kDt;
            }
            steps = march(o, d, start, bits, nullptr, 1024u);
        }
        const bool keep     = steps > 0 && base + steps <= sample_limit;
        numsteps[2 * i]     = keep ? steps : 0u;
        numsteps[2 * i + 1] = keep ? base : 0u;
        if (keep) march(o, d, start, bits, coords + static_cast<uint64_t>(base) * 7u, steps);
        base += steps;
    }
    return base;
}

// oracle_march_rays over `threads` host threads (CPU baseline timing): per-ray counts in
// parallel, their prefix sum, then the records in parallel; the same output.
uint32_t oracle_march_rays_mt(uint32_t n, const float* rays, const uint8_t* bits, uint32_t sample_limit, uint32_t* numsteps, float* coords,
                              int threads) {
    std::vector<uint32_t> steps(n, 0u);
    std::vector<float> start(n, 0.0f);
    parallel_for(n, threads, [&](uint32_t b, uint32_t e) {
        for (uint32_t i = b; i < e; ++i) {
            const float* q = rays + static_cast<uint64_t>(i) * 6u;
            const V3 o = {q[0], q[1], q[2]}, d = {q[3], q[4], q[5]};
            float tmin = 0.0f;
            if (!hit_cube(o, d, tmin)) continue;
            start[i] = tmin + 0.5f * kDt;
            steps[i] = march(o, d, start[i], bits, nullptr, 1024u);
        }
    }, 64);
    uint32_t base = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const bool keep     = steps[i] > 0 && base + steps[i] <= sample_limit;
        numsteps[2 * i]     = keep ? steps[i] : 0u;
        numsteps[2 * i + 1] = keep ? base : 0u;
        base += steps[i];
    }
    parallel_for(n, threads, [&](uint32_t b, uint32_t e) {
        for (uint32_t i = b; i < e; ++i) {
            if (numsteps[2 * i] == 0u) continue;
            const float* q = rays + static_cast<uint64_t>(i) * 6u;
            march({q[0], q[1], q[2]}, {q[3], q[4], q[5]}, start[i], bits, coords + static_cast<uint64_t>(numsteps[2 * i + 1]) * 7u, numsteps[2 * i]);
        }
    }, 64);
    return base;
}

// One segment of a segmented march (test oracle of ngp_march_rays_segment): ray list[k] (or k)
// marches at most min(cap, 1024 - marched) samples from t_state (or, for the first segment, from
// tmin + dt/2, the evaluation start of ngp.train.cu:613); t_out[k] = t of its last sample + dt
// when the segment's cap stopped it short of the ray's 1024-sample allowance, else -1.  The
// samples of all entries are written in entry order; returns their count.  A sequential march
// in state t after a sample at t_s continues at t_s + dt, so segments started at t_out
// concatenate to the single march (the property the segmented render relies on).
uint32_t oracle_march_segment(uint32_t n, const uint32_t* list, const float* rays, const uint8_t* bits, const float* t_state,
                              const uint32_t* marched, uint32_t cap, uint32_t* numsteps, float* coords, float* t_out) {
    uint32_t base = 0;
    for (uint32_t k = 0; k < n; ++k) {
        const uint32_t i = list != nullptr ? list[k] : k;
        const float* q   = rays + static_cast<uint64_t>(i) * 6u;
        const V3 o = {q[0], q[1], q[2]}, d = {q[3], q[4], q[5]};
        const uint32_t done  = marched != nullptr ? marched[i] : 0u;
        const uint32_t left  = 1024u - std::min(done, 1024u);
        const uint32_t limit = std::min(cap, left);
        float tmin = 0.0f, t_last = 0.0f;
        uint32_t steps = 0;
        if (limit > 0 && hit_cube(o, d, tmin)) {
            const float start = t_state != nullptr ? t_state[i] : tmin + 0.5f * kDt;
            steps             = march(o, d, start, bits, coords + static_cast<uint64_t>(base) * 7u, limit, &t_last);
        }
        numsteps[2 * k]     = steps;
        numsteps[2 * k + 1] = base;
        t_out[k]            = (steps == limit && limit > 0 && limit < left) ? t_last + kDt : -1.0f;
        base += steps;
    }
    return base;
}

// Density-grid samples (ngp.train.cu:383-424): uniform then non-uniform.
void oracle_grid_samples(uint32_t n_uniform, uint32_t n_nonuniform, uint32_t ema_step, const float* values, float* coords, uint32_t* indices) {
    for (uint32_t g = 0; g < n_uniform + n_nonuniform; ++g) {
        const bool uni   = g < n_uniform;
        const uint32_t i = uni ? g : g - n_uniform, count = uni ? n_uniform : n_nonuniform;
        const float thr  = uni ? -0.01f : 0.01f;
        Pcg rng(1337u);
        rng.advance(((static_cast<uint64_t>(ema_step) * 2ull + (uni ? 0ull : 1ull) + 1ull) << 32u) + static_cast<uint64_t>(i) * 4ull);
        uint32_t idx = 0;
        for (uint32_t j = 0; j < 10; ++j) {
            idx = static_cast<uint32_t>(((static_cast<uint64_t>(i) + static_cast<uint64_t>(ema_step) * count) * 56924617ull + j * 19349663ull + 96925573ull) %
                                        (128u * 128u * 128u));
            if (values[idx] > thr) break;
        }
        float* c   = coords + static_cast<uint64_t>(g) * 7u;
        c[0]       = (static_cast<float>(compact3(idx)) + rng.next_float()) / 128.0f;
        c[1]       = (static_cast<float>(compact3(idx >> 1)) + rng.next_float()) / 128.0f;
        c[2]       = (static_cast<float>(compact3(idx >> 2)) + rng.next_float()) / 128.0f;
        c[3]       = kDt;
        c[4] = c[5] = c[6] = 0.5f;
        indices[g] = idx;
    }
}

// EMA, mean (fp64) and bitfield (ngp.train.cu:434-474).  Returns the occupied count.
uint32_t oracle_grid_update(float* values, const float* scratch, float decay, float* mean_out, uint8_t* bits) {
    const uint32_t N = 128u * 128u * 128u;
    double sum       = 0.0;
    for (uint32_t i = 0; i < N; ++i) {
        const float v = values[i];
        values[i]     = v < 0.0f ? v : std::fmax(v * decay, scratch[i]);
        sum += std::fmax(values[i], 0.0f);
    }
    const float mean = static_cast<float>(sum / N);
    *mean_out        = mean;
    const float thr  = std::fmin(0.01f, mean);
    uint32_t count   = 0;
    for (uint32_t b = 0; b < N / 8; ++b) {
        uint32_t byte = 0;
        for (uint32_t j = 0; j < 8; ++j) byte |= values[8 * b + j] > thr ? (1u << j) : 0u;
        bits[b] = static_cast<uint8_t>(byte);
        count += __builtin_popcount(byte);
    }
    return count;
}

// Adam on fp32 gradients (ngp.train.cu:1261-1280), fp64-free restatement in fp32 with libm;
// parameters are independent, so `threads` (oracle_adam_mt) changes nothing but the time.
void oracle_adam_mt(uint32_t n, uint32_t n_mlp, float lr, float b1, float b2, float eps, float l2, float loss_scale, float* master, uint16_t* params,
                    const float* grads, float* m, float* v, uint32_t* steps, int threads) {
    parallel_for(n, threads, [&](uint32_t b, uint32_t e) {
    for (uint32_t i = b; i < e; ++i) {
        float g = grads[i] / loss_scale;
        if (i >= n_mlp && g == 0.0f) continue;
        const float w = master[i];
        if (i < n_mlp) g = std::fmaf(l2, w, g);
        m[i]             = std::fmaf(b1, m[i], (1.0f - b1) * g);
        v[i]             = std::fmaf(b2, v[i], (1.0f - b2) * (g * g));
        const uint32_t s = ++steps[i];
        const float lrt  = lr * std::sqrt(1.0f - std::pow(b2, static_cast<float>(s))) / (1.0f - std::pow(b1, static_cast<float>(s)));
        master[i]        = w - lrt * m[i] / (std::sqrt(v[i]) + eps);
        params[i]        = f2h(master[i]);
    }
    });
}

void oracle_adam(uint32_t n, uint32_t n_mlp, float lr, float b1, float b2, float eps, float l2, float loss_scale, float* master, uint16_t* params,
                 const float* grads, float* m, float* v, uint32_t* steps) {
    oracle_adam_mt(n, n_mlp, lr, b1, b2, eps, l2, loss_scale, master, params, grads, m, v, steps, 1);
}

// ---- evaluation compositing (accumulate_evaluation_loss_kernel, ngp.train.cu:676-745) ------
// Per pixel i of a tile starting at pixel_offset: front-to-back compositing of its samples
// (numsteps[2i] = count, numsteps[2i+1] = base; stop once the transmittance falls below 1e-4),
// the target read as premultiplied linear RGBA and converted back to sRGB (ngp.train.cu:264-293),
// both clamped to [0, 1]; the fp64 squared error is summed in pixel order into *sse, and the
// comparison image [height][2*width][3] (target left, render right) is written when given.
// exp / pow come from libm (the reference uses the device's expf, __expf and powf), so results
// agree with the GPU to a few ulp per operation, not bit for bit.
namespace {
inline float sigmoid_ref(float x) { return 1.0f / (1.0f + std::exp(-x)); }
inline float srgb_to_linear_ref(float v) { return v <= 0.04045f ? v / 12.92f : std::pow((v + 0.055f) / 1.055f, 2.4f); }
inline float linear_to_srgb_ref(float v) { return v < 0.0031308f ? 12.92f * v : std::fmaf(1.055f, std::pow(v, 0.41666f), -0.055f); }
inline float clamp01(float v) { return std::fmin(std::fmax(v, 0.0f), 1.0f); }
}  // namespace

void oracle_eval_composite(uint32_t tile_pixels, uint32_t pixel_offset, uint32_t image, uint32_t width, uint32_t height, const uint8_t* pixels,
                           const uint32_t* numsteps, const float* coords, const uint16_t* network_output, double* sse, uint8_t* comparison) {
    double total = 0.0;
    for (uint32_t i = 0; i < tile_pixels; ++i) {
        const uint32_t gp = pixel_offset + i, px = gp % width, py = gp / width;
        const uint32_t count = numsteps[2u * i], base = numsteps[2u * i + 1u];
        float T = 1.0f, rgb[3] = {0.0f, 0.0f, 0.0f};
        for (uint32_t j = 0; j < count; ++j) {
            const uint16_t* o   = network_output + (static_cast<uint64_t>(base) + j) * 16u;
            const float dt      = coords[(static_cast<uint64_t>(base) + j) * 7u + 3u];
            const float density = std::exp(h2f(o[3]));
            const float alpha   = 1.0f - std::exp(-density * dt);
            const float weight  = alpha * T;
            for (int c = 0; c < 3; ++c) rgb[c] = std::fmaf(weight, sigmoid_ref(h2f(o[c])), rgb[c]);
            T *= 1.0f - alpha;
            if (T < 1e-4f) break;
        }
        const uint8_t* t8 = pixels + 4u * (px + static_cast<uint64_t>(py) * width + static_cast<uint64_t>(image) * width * height);
        const float a     = static_cast<float>(t8[3]) * (1.0f / 255.0f);
        float target[3], pred[3];
        for (int c = 0; c < 3; ++c) {
            const float lin = srgb_to_linear_ref(static_cast<float>(t8[c]) * (1.0f / 255.0f)) * a;
            target[c]       = clamp01(linear_to_srgb_ref(lin));
            pred[c]         = clamp01(rgb[c]);
            const double d  = static_cast<double>(pred[c]) - static_cast<double>(target[c]);
            total += d * d;
        }
        if (comparison != nullptr) {
            const uint64_t row = static_cast<uint64_t>(py) * width * 6u;
            for (int c = 0; c < 3; ++c) {
                comparison[row + px * 3u + c]                                      = static_cast<uint8_t>(target[c] * 255.0f + 0.5f);
                comparison[row + (static_cast<uint64_t>(width) + px) * 3u + c] = static_cast<uint8_t>(pred[c] * 255.0f + 0.5f);
            }
        }
    }
    *sse += total;
}

// ---- seeded initialisation (ngp.train.cu:1002-1017, 1423-1490) -----------------------------
// master[0, 10240): the MLP matrices in packed order (density W_in 64x32, W_out 16x64, rgb W_in
// 64x32, W_h 64x64, W_out 16x64), each Xavier-uniform with scale sqrt(6 / (fan_in + fan_out)),
// drawn one after another from one PCG32(1337) stream (initialize_mlp_parameters).
// master[10240, 10240 + n_grid): U(-1e-4, 1e-4) grid entries; thread slot i of the reference's
// launch (n_slots = ceil(ceil(n_grid / 4) / 128) * 128 threads) continues the stream after the
// MLP's 10240 draws at offset 4i and writes entries i + n_slots * j, j < 4
// (initialize_grid_params_kernel).  params = fp16 of master (round to nearest even).
void oracle_init_params(uint32_t n_grid, float* master, uint16_t* params) {
    const uint32_t shapes[5][2] = {{64, 32}, {16, 64}, {64, 32}, {64, 64}, {16, 64}};
    Pcg rng(1337u);
    uint32_t off = 0;
    for (const auto& sh : shapes) {
        const float scale = std::sqrt(6.0f / static_cast<float>(sh[0] + sh[1]));
        for (uint32_t i = 0; i < sh[0] * sh[1]; ++i) {
            const float u    = rng.next_float() * 2.0f;
            master[off + i] = u * scale - scale;
        }
        off += sh[0] * sh[1];
    }
    const uint32_t slots = (((n_grid + 3u) / 4u + 127u) / 128u) * 128u;
    for (uint32_t i = 0; i < slots; ++i) {
        Pcg g(1337u);
        g.advance(10240ull + 4ull * i);
        for (uint32_t j = 0; j < 4; ++j) {
            const uint64_t idx = i + static_cast<uint64_t>(slots) * j;
            if (idx >= n_grid) break;
            master[off + idx] = std::fmaf(g.next_float(), 2e-4f, -1e-4f);
        }
    }
    for (uint32_t i = 0; i < off + n_grid; ++i) params[i] = f2h(master[i]);
}

}  // extern "C"
