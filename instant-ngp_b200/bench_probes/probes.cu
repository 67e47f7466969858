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
