// Bench-only throughput probes (not part of libngp_b200.so): the denominators of the encoding
// kernels' L2 roofline, measured on the GPU that runs the benchmark.
//
//  * probe_l2_read: streaming 16-byte loads over an L2-resident buffer, many passes — the L2
//    read bandwidth a kernel whose working set fits in L2 can reach.
//  * probe_gather: random 4-byte loads from an L2-resident table, 16 independent loads per
//    thread per round (as the hash-grid kernels issue 16 levels x 8 corners per point).
//  * probe_scatter: random float2 atomic adds into an L2-resident table.
//
// Built by instant-ngp_b200/build.py into bench_probes/libngp_bench_probes.so; loaded only by
// bench.py.  Return value: a cudaError_t (0 = success).
#include <cuda_runtime.h>

#include <cstdint>

namespace {

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16, x *= 0x7feb352du, x ^= x >> 15, x *= 0x846ca68bu, x ^= x >> 16;
    return x;
}

__global__ void __launch_bounds__(256) l2_read_kernel(const uint4* __restrict__ buf, uint32_t n_vec, uint32_t passes, uint32_t* __restrict__ out) {
    const uint32_t stride = gridDim.x * blockDim.x;
    uint32_t acc          = 0;
    for (uint32_t p = 0; p < passes; ++p) {
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n_vec; i += 4 * stride) {
            uint4 v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint32_t j = i + k * stride;
                v[k]             = j < n_vec ? __ldcg(buf + j) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) acc ^= v[k].x + v[k].y + v[k].z + v[k].w;
        }
    }
    if (acc == 0x12345678u) out[0] = acc;  // keeps the loads alive
}

__global__ void __launch_bounds__(256) gather_probe_kernel(const uint32_t* __restrict__ table, uint32_t mask, uint32_t rounds, uint32_t* __restrict__ out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t acc = 0, h = mix32(i);
    for (uint32_t r = 0; r < rounds; ++r) {
        uint32_t v[16];
#pragma unroll
        for (uint32_t k = 0; k < 16; ++k) v[k] = __ldg(table + (mix32(h + k) & mask));
#pragma unroll
        for (uint32_t k = 0; k < 16; ++k) acc += v[k];
        h = mix32(h ^ acc);
    }
    out[i] = acc;
}

__global__ void __launch_bounds__(256) scatter_probe_kernel(float2* __restrict__ table, uint32_t mask, uint32_t rounds) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t h       = mix32(i);
    for (uint32_t r = 0; r < rounds; ++r) {
#pragma unroll
        for (uint32_t k = 0; k < 16; ++k) atomicAdd(table + (mix32(h + k) & mask), make_float2(1.0f, 1.0f));
        h = mix32(h + 0x9e3779b9u);
    }
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int probe_l2_read(const void* buf, size_t bytes, uint32_t passes, uint32_t* out, void* stream) {
    if (buf == nullptr || out == nullptr || bytes < 16 || bytes % 16 != 0 || bytes / 16 > 0xFFFFFFFFull) return cudaErrorInvalidValue;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    l2_read_kernel<<<sms * 8, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint4*>(buf), static_cast<uint32_t>(bytes / 16), passes, out);
    return cudaGetLastError();
}

extern "C" __attribute__((visibility("default"))) int probe_gather(const uint32_t* table, uint32_t log2_entries, uint32_t threads, uint32_t rounds,
                                                                    uint32_t* out, void* stream) {
    if (table == nullptr || out == nullptr || threads == 0 || threads % 256u != 0 || log2_entries > 31) return cudaErrorInvalidValue;
    gather_probe_kernel<<<threads / 256u, 256, 0, static_cast<cudaStream_t>(stream)>>>(table, (1u << log2_entries) - 1u, rounds, out);
    return cudaGetLastError();
}

extern "C" __attribute__((visibility("default"))) int probe_scatter(float* table, uint32_t log2_entries, uint32_t threads, uint32_t rounds, void* stream) {
    if (table == nullptr || threads == 0 || threads % 256u != 0 || log2_entries > 31) return cudaErrorInvalidValue;
    scatter_probe_kernel<<<threads / 256u, 256, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<float2*>(table), (1u << log2_entries) - 1u,
                                                                                       rounds);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------------------------
// tcgen05 MMA issue rate: each CTA's thread 0 issues `count` dependent-accumulate MMAs of shape
// M = 128, N = n, K = 16 (fp16 in, fp32 TMEM accumulator) from shared-memory tiles, commits them
// to an mbarrier and waits (bounded); the kernel time / count gives the cost of one instruction.
// ---------------------------------------------------------------------------------------------
#include "umma.cuh"

namespace {
__global__ void __launch_bounds__(128) mma_rate_kernel(uint32_t n, uint32_t count, uint32_t* status) {
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ uint64_t mbar;
    __shared__ uint32_t tmem_slot;
    for (uint32_t i = threadIdx.x; i < (128u * 16u + 256u * 16u) * 2u / 16u; i += blockDim.x) reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x < 32) ngp::umma::tmem_alloc(&tmem_slot, 256);
    if (threadIdx.x == 0) ngp::umma::mbar_init(&mbar, 1);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    ngp::umma::fence_before_sync();
    __syncthreads();
    ngp::umma::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    if (threadIdx.x == 0) {
        const uint32_t a = ngp::umma::smem_addr(smem), b = a + 128u * 16u * 2u;
        const uint64_t ad = ngp::umma::make_desc(a, 128u, 256u), bd = ngp::umma::make_desc(b, 128u, 256u);
        const uint32_t idesc = ngp::umma::make_idesc_f16(128u, n, false, false);
        for (uint32_t k = 0; k < count; ++k) ngp::umma::mma_f16(tmem, ad, bd, idesc, k > 0 ? 1u : 0u);
        ngp::umma::commit(&mbar);
    }
    const bool ok = ngp::umma::mbar_wait(&mbar, 0);
    if (!ok && threadIdx.x == 0) atomicOr(status, 1u);
    ngp::umma::fence_after_sync();
    __syncthreads();
    if (threadIdx.x < 32) ngp::umma::tmem_dealloc(tmem, 256);
}
}  // namespace

extern "C" __attribute__((visibility("default"))) int probe_mma_rate(uint32_t n, uint32_t count, uint32_t ctas, uint32_t* status, void* stream) {
    if (n < 16 || n > 256 || n % 16 != 0 || count == 0 || ctas == 0 || status == nullptr) return cudaErrorInvalidValue;
    const int smem = (128 * 16 + 256 * 16) * 2;
    mma_rate_kernel<<<ctas, 128, smem, static_cast<cudaStream_t>(stream)>>>(n, count, status);
    return cudaGetLastError();
}

// Dependent chain of `iters` stages, as one layer of the fused MLPs: thread 0 issues `k` MMAs
// (M = 128, N = n, K = 16) and commits; every thread waits for the mbarrier, reads 64 fp32
// columns of its TMEM lane, writes 128 bytes of its row back to shared memory (the next layer's
// operand) and the CTA synchronises.  Kernel time / iters = one stage's latency.
namespace {
__global__ void __launch_bounds__(128) mma_chain_kernel(uint32_t n, uint32_t k, uint32_t iters, uint32_t* status) {
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ uint64_t mbar;
    __shared__ uint32_t tmem_slot;
    for (uint32_t i = threadIdx.x; i < (128u * 64u + 256u * 64u) * 2u / 16u; i += blockDim.x) reinterpret_cast<uint4*>(smem)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x < 32) ngp::umma::tmem_alloc(&tmem_slot, 256);
    if (threadIdx.x == 0) ngp::umma::mbar_init(&mbar, 1);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    ngp::umma::fence_before_sync();
    __syncthreads();
    ngp::umma::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    const uint32_t a = ngp::umma::smem_addr(smem), b = a + 128u * 64u * 2u;
    uint32_t phase = 0;
    float acc      = 0.0f;
    for (uint32_t it = 0; it < iters; ++it) {
        if (threadIdx.x == 0) {
            const uint32_t idesc = ngp::umma::make_idesc_f16(128u, n, false, false);
            for (uint32_t q = 0; q < k; ++q)
                ngp::umma::mma_f16(tmem, ngp::umma::make_desc(a + q * 256u, 128u, 1024u), ngp::umma::make_desc(b + q * 256u, 128u, 1024u), idesc,
                                   q > 0 ? 1u : 0u);
            ngp::umma::commit(&mbar);
        }
        if (!ngp::umma::mbar_wait(&mbar, phase)) atomicOr(status, 1u);
        phase ^= 1u;
        ngp::umma::fence_after_sync();
        uint32_t r[4][16];
        const uint32_t lane_base = (threadIdx.x & ~31u) << 16;
#pragma unroll
        for (uint32_t c = 0; c < 4; ++c) ngp::umma::tmem_ld16_async(tmem + lane_base + c * 16u, r[c]);
        ngp::umma::tmem_wait_ld();
        uint4 v[4];
#pragma unroll
        for (uint32_t c = 0; c < 4; ++c) v[c] = make_uint4(r[c][0] & 0u, r[c][1] & 0u, r[c][2] & 0u, r[c][3] & 0u), acc += __uint_as_float(r[c][5]);
        uint4* row = reinterpret_cast<uint4*>(smem + (threadIdx.x & 7u) * 16u + (threadIdx.x >> 3) * 1024u);
#pragma unroll
        for (uint32_t c = 0; c < 4; ++c) row[c * 8] = v[c];
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        ngp::umma::fence_before_sync();
        __syncthreads();
        ngp::umma::fence_after_sync();
    }
    if (acc == 12345.0f) atomicOr(status, 2u);
    __syncthreads();
    if (threadIdx.x < 32) ngp::umma::tmem_dealloc(tmem, 256);
}
}  // namespace

extern "C" __attribute__((visibility("default"))) int probe_mma_chain(uint32_t n, uint32_t k, uint32_t iters, uint32_t ctas, uint32_t* status,
                                                                       void* stream) {
    if (n < 16 || n > 256 || n % 16 != 0 || k == 0 || k > 4 || iters == 0 || ctas == 0 || status == nullptr) return cudaErrorInvalidValue;
    const int smem = (128 * 64 + 256 * 64) * 2;
    if (const cudaError_t e = cudaFuncSetAttribute(mma_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); e != cudaSuccess) return e;
    mma_chain_kernel<<<ctas, 128, smem, static_cast<cudaStream_t>(stream)>>>(n, k, iters, status);
    return cudaGetLastError();
}
