// Throughput probes for the roofline of the gather / scatter-bound kernels: the rate of random
// 4-byte loads from (and 2 x fp32 atomic adds into) an L2-resident table on this GPU, measured by
// the benchmark beside the kernels it bounds.  Each thread of the gather probe issues 16
// independent loads per round from pseudo-random entries (a 32-bit integer hash of its index),
// as the hash-grid kernels do (16 levels x 8 corners per point, in flight two levels at a time).
#include "common.cuh"

namespace ngp {
namespace {

__device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16, x *= 0x7feb352du, x ^= x >> 15, x *= 0x846ca68bu, x ^= x >> 16;
    return x;
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
}  // namespace ngp

using namespace ngp;

extern "C" int ngp_probe_gather(const uint32_t* table, uint32_t log2_entries, uint32_t threads, uint32_t rounds, uint32_t* out, void* stream) {
    clear_error();
    if (table == nullptr || out == nullptr || threads == 0 || threads % 256u != 0 || log2_entries > 31)
        return fail(NGP_ERR_INVALID, "gather probe: invalid input");
    gather_probe_kernel<<<threads / 256u, 256, 0, as_stream(stream)>>>(table, (1u << log2_entries) - 1u, rounds, out);
    return check_launch("gather_probe_kernel");
}

extern "C" int ngp_probe_scatter(float* table, uint32_t log2_entries, uint32_t threads, uint32_t rounds, void* stream) {
    clear_error();
    if (table == nullptr || threads == 0 || threads % 256u != 0 || log2_entries > 31) return fail(NGP_ERR_INVALID, "scatter probe: invalid input");
    scatter_probe_kernel<<<threads / 256u, 256, 0, as_stream(stream)>>>(reinterpret_cast<float2*>(table), (1u << log2_entries) - 1u, rounds);
    return check_launch("scatter_probe_kernel");
}
