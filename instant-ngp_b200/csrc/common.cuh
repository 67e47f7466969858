// Shared helpers for the sm_100a kernels: status handling, launch geometry, the hash-grid
// index math and the reference's PCG32 generator.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "ngp_b200.h"

namespace ngp {

// ---- status --------------------------------------------------------------------------------
void set_error(const std::string& message);
void clear_error();

inline int fail(int code, const std::string& message) {
    set_error(message);
    return code;
}

void count_launch();

// Host-side fault injection (ngp_fault_inject / $NGP_FAULT_INJECT): true when the armed
// countdown of `site` reaches this event, which then reports an error instead of its result.
// No device code is involved: the injected failure is a status the host returns.
enum FaultSite : int { kFaultAlloc = 1, kFaultLaunch = 2, kFaultCollective = 3 };
bool fault_due(FaultSite site);

// Called once after every kernel launch of the library (also counts it).
inline int check_launch(const char* what) {
    count_launch();
    if (fault_due(kFaultLaunch)) {
        (void)cudaGetLastError();
        return fail(NGP_ERR_CUDA, std::string(what) + ": injected fault (launch)");
    }
    const cudaError_t status = cudaGetLastError();
    if (status != cudaSuccess) return fail(NGP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(status));
    return NGP_OK;
}

inline int check_cuda(cudaError_t status, const char* what) {
    if (status != cudaSuccess) return fail(NGP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(status));
    return NGP_OK;
}

#define NGP_TRY(expr)                        \
    do {                                     \
        const int ngp_status_ = (expr);      \
        if (ngp_status_ != NGP_OK) return ngp_status_; \
    } while (0)

inline cudaStream_t as_stream(void* stream) { return static_cast<cudaStream_t>(stream); }

// Encoded-feature buffers: feature-major [features][stride] (the reference's layout) or, with
// NGP_ROWS set in the stride argument, row-major [rows][features].
__host__ __device__ inline bool rows_layout(uint32_t stride) { return (stride & NGP_ROWS) != 0u; }

// Number of SMs of the current device (148 on B200), cached per process.
int sm_count();

// Data-parallel gradient exchange fused with Adam over NVLink peer memory (adam.cu): every rank
// reads the fp16 gradients of its parameter shard from all ranks' buffers, sums them in rank
// order, takes the Adam step on its shard and writes the new fp16 parameters into every rank's
// parameter buffer.  Cross-GPU ordering uses per-rank flag words in peer memory (an arrival
// barrier before the reads, a completion barrier after the writes), each wait bounded in time.
struct PeerExchangeArgs {
    uint32_t rank, world, shard, n_params, n_mlp, epoch;
    float lr, beta1, beta2, eps, l2, loss_scale;
    const __half* const* grads;  // [world] device pointers (this rank's entry: its own buffer)
    __half* const* params;       // [world]
    uint32_t* const* flags;      // [world]: 2 * world flag words + one CTA counter each
    float* master;
    float* m;
    float* v;
    uint32_t* steps;
    const float* lr_table;
    uint32_t table_len;
    uint32_t* status;  // bit 0: arrival wait timed out, bit 1: completion wait timed out
};
int peer_exchange_adam(const PeerExchangeArgs& a, cudaStream_t stream);

// ---- hash grid -----------------------------------------------------------------------------
// Kernel-parameter copy of ngp_grid_layout (only what the device needs).
struct GridParams {
    uint32_t n_levels;
    uint32_t dense_mask;  // bit l: level l is dense-indexed (r <= 0x659 and r^3 <= its size)
    uint32_t offsets[NGP_MAX_LEVELS + 1];
    uint32_t resolution[NGP_MAX_LEVELS];
    float scale[NGP_MAX_LEVELS];
};

inline GridParams make_grid_params(const ngp_grid_layout& layout) {
    GridParams p{};
    p.n_levels = layout.n_levels;
    for (uint32_t l = 0; l <= layout.n_levels; ++l) p.offsets[l] = layout.offsets[l];
    for (uint32_t l = 0; l < layout.n_levels; ++l) {
        p.resolution[l] = layout.resolution[l];
        p.scale[l]      = layout.scale[l];
        const uint32_t r = layout.resolution[l], size = layout.offsets[l + 1] - layout.offsets[l];
        if (r <= 0x659u && r * r * r <= size) p.dense_mask |= 1u << l;
    }
    return p;
}

// Grid index of corner (x, y, z): dense x + y*r + z*r^2 while r <= 0x659 and r^3 fits the
// level, otherwise the spatial hash x ^ y*2654435761 ^ z*805459861; then modulo the level size.
// Same integer function as the reference's grid_index / coherent_prime_hash
// (ngp.train.cu:165-186), which must be reproduced bit for bit.
__device__ __forceinline__ uint32_t grid_index(uint32_t hashmap_size, uint32_t resolution, uint32_t x,
                                               uint32_t y, uint32_t z) {
    uint32_t index;
    uint32_t stride;
    if (resolution <= 0x659u) {
        index  = x + y * resolution + z * (resolution * resolution);
        stride = resolution * resolution * resolution;
    } else {
        index  = 0u;
        stride = 0xFFFFFFFFu;
    }
    if (hashmap_size < stride) index = x ^ (y * 2654435761u) ^ (z * 805459861u);
    // index % hashmap_size without the integer division where it is not needed: hashed levels
    // have a power-of-two size (a mask), and dense indices are below the size except for the
    // +1 corners on the upper faces
    if ((hashmap_size & (hashmap_size - 1u)) == 0u) return index & (hashmap_size - 1u);
    return index < hashmap_size ? index : index % hashmap_size;
}

// The 8 corner indices of cell (x, y, z) at one level, corner c = x bit 0, y bit 1, z bit 2:
// grid_index specialised by the level's kind, which is uniform across a warp.  Dense levels:
// x + y*r + z*r^2 is below 2 * size for points in [0, 1] (size >= r^3 and the +1 corners add at
// most r^2 + r + 1), so the modulo is one conditional subtraction; hashed levels have a power-of-two size (a mask).
__device__ __forceinline__ void corner_indices(bool dense, uint32_t size, uint32_t r, uint32_t x, uint32_t y, uint32_t z, uint32_t (&idx)[8]) {
    if (dense) {
        const uint32_t r2 = r * r, base = x + y * r + z * r2;
#pragma unroll
        for (uint32_t c = 0; c < 8; ++c) {
            const uint32_t i = base + (c & 1u) + ((c >> 1) & 1u) * r + (c >> 2) * r2;
            idx[c]           = i < size ? i : (i - size < size ? i - size : i % size);  // the last case only for points outside [0, 1]
        }
    } else {
        const uint32_t hy[2] = {y * 2654435761u, (y + 1u) * 2654435761u};
        const uint32_t hz[2] = {z * 805459861u, (z + 1u) * 805459861u};
        const uint32_t mask  = size - 1u;
#pragma unroll
        for (uint32_t c = 0; c < 8; ++c) idx[c] = ((x + (c & 1u)) ^ hy[(c >> 1) & 1u] ^ hz[c >> 2]) & mask;
    }
}

// ---- PCG32 ---------------------------------------------------------------------------------
// The reference's PCG32 (ngp.train.cu:85-143): O'Neill's pcg32 (XSH-RR 64/32) with the
// default stream constants and the LCG jump-ahead of Brown (1994).  All training randomness
// must follow it exactly so that sample positions are bit-identical to the reference's.
// Jump table of the default stream (inc = 3): advancing the state by 2^k steps is the affine map
// state -> mult[k] * state + plus[k] (mod 2^64).  Composing the maps of delta's set bits gives the
// same state as Brown's loop below (LCG steps commute), with one multiply-add per set bit.
struct PcgJumpTable {
    uint64_t mult[64];
    uint64_t plus[64];
};

constexpr PcgJumpTable make_pcg_jump_table() {
    PcgJumpTable t{};
    uint64_t m = 0x5851f42d4c957f2dULL, c = 3u;
    for (int k = 0; k < 64; ++k) {
        t.mult[k] = m;
        t.plus[k] = c;
        c         = (m + 1u) * c;
        m *= m;
    }
    return t;
}

static __constant__ PcgJumpTable c_pcg_jump = make_pcg_jump_table();

struct Pcg32 {
    uint64_t state;
    uint64_t inc;

    __host__ __device__ explicit Pcg32(uint64_t initstate, uint64_t initseq = 1u) {
        state = 0u;
        inc   = (initseq << 1u) | 1u;
        next_uint();
        state += initstate;
        next_uint();
    }
    __host__ __device__ uint32_t next_uint() {
        const uint64_t old = state;
        state              = old * 0x5851f42d4c957f2dULL + inc;
        const uint32_t xs  = static_cast<uint32_t>(((old >> 18u) ^ old) >> 27u);
        const uint32_t rot = static_cast<uint32_t>(old >> 59u);
        return (xs >> rot) | (xs << ((~rot + 1u) & 31u));
    }
    __host__ __device__ float next_float() {
        const uint32_t bits = (next_uint() >> 9u) | 0x3f800000u;
        float value;
        memcpy(&value, &bits, sizeof(value));
        return value - 1.0f;
    }
    __host__ __device__ void advance(uint64_t delta) {
#ifdef __CUDA_ARCH__
        if (inc == 3u) {
            while (delta != 0u) {
                const int k = __ffsll(static_cast<long long>(delta)) - 1;
                state       = c_pcg_jump.mult[k] * state + c_pcg_jump.plus[k];
                delta &= delta - 1u;
            }
            return;
        }
#endif
        uint64_t cur_mult = 0x5851f42d4c957f2dULL, cur_plus = inc, acc_mult = 1u, acc_plus = 0u;
        while (delta > 0u) {
            if (delta & 1u) {
                acc_mult *= cur_mult;
                acc_plus = acc_plus * cur_mult + cur_plus;
            }
            cur_plus = (cur_mult + 1u) * cur_plus;
            cur_mult *= cur_mult;
            delta >>= 1u;
        }
        state = acc_mult * state + acc_plus;
    }
};

constexpr uint64_t kTrainSeed = 1337u;

}  // namespace ngp
