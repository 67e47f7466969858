// ref_harness.cu -- builds the REFERENCE implementation (Xayah-Graphics/instant-ngp
// ngp.train.cu, unmodified, included from its own source tree at build time) into
// oracle/_ref/libngp_ref.so and exposes its kernels through a small extern "C" surface.
//
// TEST INFRASTRUCTURE ONLY: used by tests/ (golden fixtures, GPU parity) and by bench.py's
// reference arm.  Nothing in the product links or loads it.  Compiled for sm_100a by
// oracle/Makefile; the reference's own source is never copied into this repository.
//
// The reference's kernels live in an anonymous namespace inside ngp::cuda; including the
// translation unit here makes them callable from the wrappers below, launched with the
// reference's own launch shapes (ngp.train.cu:1506-1507, 1899-1901).
#include "ngp.train.cu"

namespace ref = ngp::cuda;
namespace cfg = ngp::cuda::config;

namespace {
int status_of(cudaError_t e) { return e == cudaSuccess ? 0 : static_cast<int>(e); }
}  // namespace

extern "C" {

// Grid offsets of the reference layout (8 levels x 4 features, ngp.train.h:44-56).
int ref_grid_offsets(uint32_t* out9) {
    for (uint32_t l = 0; l <= cfg::GRID_N_LEVELS; ++l) out9[l] = cfg::NETWORK_PARAMETER_LAYOUT.grid_offsets[l];
    return 0;
}

uint32_t ref_total_param_count() { return cfg::NETWORK_PARAMETER_LAYOUT.total_param_count; }
uint32_t ref_mlp_param_count() { return cfg::NETWORK_PARAMETER_LAYOUT.mlp_param_count; }

// encode_grid_forward_kernel (ngp.train.cu:876-921) on n points of 7-float sample records.
int ref_encode_forward(uint32_t n, const float* coords, const uint16_t* grid, uint16_t* out, void* stream) {
    const auto& L = cfg::NETWORK_PARAMETER_LAYOUT;
    const dim3 blocks{(n + ref::GRID_FORWARD_THREADS - 1u) / ref::GRID_FORWARD_THREADS, cfg::GRID_N_LEVELS, 1u};
    ref::encode_grid_forward_kernel<<<blocks, ref::GRID_FORWARD_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        n, L.grid_offsets[0], L.grid_offsets[1], L.grid_offsets[2], L.grid_offsets[3], L.grid_offsets[4], L.grid_offsets[5],
        L.grid_offsets[6], L.grid_offsets[7], L.grid_offsets[8], coords, reinterpret_cast<const __half*>(grid),
        reinterpret_cast<__half*>(out));
    return status_of(cudaGetLastError());
}

// encode_grid_backward_kernel (ngp.train.cu:923-960): fp16 half2 atomics into grad (not zeroed).
int ref_encode_backward(uint32_t n, const float* coords, const uint16_t* dy, uint16_t* grad, void* stream) {
    const auto& L           = cfg::NETWORK_PARAMETER_LAYOUT;
    const uint32_t threads  = (n * cfg::GRID_FEATURES_PER_LEVEL / ref::GRID_BACKWARD_FEATURES + ref::GRID_BACKWARD_THREADS - 1u) / ref::GRID_BACKWARD_THREADS;
    const dim3 blocks{threads, cfg::GRID_N_LEVELS, 1u};
    ref::encode_grid_backward_kernel<<<blocks, ref::GRID_BACKWARD_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
        n, L.grid_offsets[0], L.grid_offsets[1], L.grid_offsets[2], L.grid_offsets[3], L.grid_offsets[4], L.grid_offsets[5],
        L.grid_offsets[6], L.grid_offsets[7], L.grid_offsets[8], coords, reinterpret_cast<const __half*>(dy),
        reinterpret_cast<__half*>(grad));
    return status_of(cudaGetLastError());
}

// encode_spherical_harmonics_kernel (ngp.train.cu:962-993) -> fp16 [16][n].
int ref_sh_encode(uint32_t n, const float* coords, uint16_t* out, void* stream) {
    ref::encode_spherical_harmonics_kernel<<<(n + ref::THREADS_PER_BLOCK - 1u) / ref::THREADS_PER_BLOCK, ref::THREADS_PER_BLOCK, 0,
                                             static_cast<cudaStream_t>(stream)>>>(n, coords, reinterpret_cast<__half*>(out));
    return status_of(cudaGetLastError());
}

// The reference's two MLP launches and density extraction of evaluate_network
// (ngp.train.cu:1514-1522) on a given encoded input x [32][n] and SH block sh [16][n]:
// density net -> rgb_in[0..15], rgb net -> out [n][16], out[:,3] = density.  n % 128 == 0.
int ref_mlp_forward(uint32_t n, const uint16_t* mlp_params, const uint16_t* x, uint16_t* rgb_in, uint16_t* out, void* stream) {
    const auto s                 = static_cast<cudaStream_t>(stream);
    constexpr int forward_shmem  = sizeof(__half) * (16u + 16u * ref::MLP_FORWARD_ITERS) * (cfg::MLP_WIDTH + ref::MLP_SKEW);
    constexpr dim3 threads{32u, ref::MLP_WIDTH_BLOCKS, 1u};
    if (cudaFuncSetAttribute(ref::mlp_forward_64_relu_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, forward_shmem) != cudaSuccess) return 1;
    const dim3 blocks{n / (16u * ref::MLP_FORWARD_ITERS), 1u, 1u};
    const auto* P = reinterpret_cast<const __half*>(mlp_params);
    ref::mlp_forward_64_relu_kernel<<<blocks, threads, forward_shmem, s>>>(n, reinterpret_cast<const __half*>(x), P + cfg::NETWORK_PARAMETER_LAYOUT.density_param_offset,
                                                                           nullptr, reinterpret_cast<__half*>(rgb_in), false, cfg::DENSITY_HIDDEN_LAYERS);
    ref::mlp_forward_64_relu_kernel<<<blocks, threads, forward_shmem, s>>>(n, reinterpret_cast<const __half*>(rgb_in), P + cfg::NETWORK_PARAMETER_LAYOUT.rgb_param_offset,
                                                                           nullptr, reinterpret_cast<__half*>(out), true, cfg::RGB_HIDDEN_LAYERS);
    ref::extract_density_kernel<<<(n + ref::THREADS_PER_BLOCK - 1u) / ref::THREADS_PER_BLOCK, ref::THREADS_PER_BLOCK, 0, s>>>(
        n, reinterpret_cast<const __half*>(rgb_in), reinterpret_cast<__half*>(out));
    return status_of(cudaGetLastError());
}

// PCG32 as the reference's device code runs it (ngp.train.cu:89-143), for pinning.
int ref_pcg32(uint64_t initstate, uint64_t initseq, uint64_t advance, uint32_t count, uint32_t* out_uint, float* out_float) {
    ref::Pcg32 a{initstate, initseq};
    a.advance(advance);
    ref::Pcg32 b = a;
    for (uint32_t i = 0; i < count; ++i) {
        out_uint[i]  = a.next_uint();
        out_float[i] = b.next_float();
    }
    return 0;
}

}  // extern "C"
