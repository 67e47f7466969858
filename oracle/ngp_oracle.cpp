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
