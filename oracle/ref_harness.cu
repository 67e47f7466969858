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

// generate_training_samples_kernel (ngp.train.cu:476-578), counters cleared first.
int ref_generate_training_samples(uint32_t rays_per_batch, uint32_t sample_limit, uint32_t step, uint32_t frame_count, uint32_t width,
                                  uint32_t height, float fx, float fy, float cx, float cy, const float* camera, const uint8_t* occupancy,
                                  uint32_t* ray_counter, uint32_t* sample_counter, uint32_t* ray_indices, float* rays, uint32_t* numsteps,
                                  float* coords) {
    cudaMemset(ray_counter, 0, 4);
    cudaMemset(sample_counter, 0, 4);
    ref::generate_training_samples_kernel<<<(rays_per_batch + 127u) / 128u, 128u>>>(rays_per_batch, sample_limit, step, frame_count, width, height, fx,
                                                                                     fy, cx, cy, camera, occupancy, ray_counter, sample_counter,
                                                                                     ray_indices, rays, numsteps, coords);
    return status_of(cudaDeviceSynchronize());
}

// generate_evaluation_samples_kernel (ngp.train.cu:580-667) for one tile of pixels.
int ref_generate_evaluation_samples(uint32_t tile_pixels, uint32_t pixel_offset, uint32_t max_samples, uint32_t width, uint32_t height, float fx,
                                    float fy, float cx, float cy, const float* camera, uint32_t image, const uint8_t* occupancy,
                                    uint32_t* sample_counter, uint32_t* overflow_counter, uint32_t* numsteps, float* coords) {
    cudaMemset(sample_counter, 0, 4);
    cudaMemset(overflow_counter, 0, 4);
    ref::generate_evaluation_samples_kernel<<<(tile_pixels + 127u) / 128u, 128u>>>(tile_pixels, pixel_offset, max_samples, width, height, fx, fy, cx,
                                                                                   cy, camera, image, occupancy, sample_counter, overflow_counter,
                                                                                   numsteps, coords);
    return status_of(cudaDeviceSynchronize());
}

// mark_untrained_density_grid_kernel (ngp.train.cu:310-381).
int ref_mark_untrained(float* values, uint32_t frame_count, uint32_t width, uint32_t height, float fx, float fy, float cx, float cy,
                       const float* camera) {
    ref::mark_untrained_density_grid_kernel<<<ref::NERF_GRID_CELLS / 128u, 128u>>>(values, frame_count, width, height, fx, fy, cx, cy, camera);
    return status_of(cudaDeviceSynchronize());
}

// generate_density_grid_samples_kernel (ngp.train.cu:383-424), uniform (phase 0) then nonuniform.
int ref_grid_samples(uint32_t n_uniform, uint32_t n_nonuniform, uint32_t ema_step, const float* values, float* coords, uint32_t* indices) {
    if (n_uniform)
        ref::generate_density_grid_samples_kernel<<<(n_uniform + 127u) / 128u, 128u>>>(n_uniform, ema_step, 0u, -0.01f, values, coords, indices);
    if (n_nonuniform)
        ref::generate_density_grid_samples_kernel<<<(n_nonuniform + 127u) / 128u, 128u>>>(n_nonuniform, ema_step, 1u, ref::NERF_MIN_OPTICAL_THICKNESS,
                                                                                          values, coords + static_cast<uint64_t>(n_uniform) * 7u,
                                                                                          indices + n_uniform);
    return status_of(cudaDeviceSynchronize());
}

// K3-K6 (ngp.train.cu:426-474): splat, EMA, mean, bitfield, in the reference's launch order.
int ref_grid_update(uint32_t n, const uint32_t* indices, const uint16_t* density, float* scratch, float* values, float* mean, uint8_t* occupancy,
                    uint32_t* occupied) {
    ref::splat_density_grid_samples_kernel<<<(n + 127u) / 128u, 128u>>>(n, indices, reinterpret_cast<const __half*>(density), scratch);
    ref::update_density_grid_ema_kernel<<<ref::NERF_GRID_CELLS / 128u, 128u>>>(scratch, values);
    cudaMemset(mean, 0, 4);
    cudaMemset(occupied, 0, 4);
    ref::reduce_density_grid_mean_kernel<<<(ref::NERF_GRID_CELLS / 4u + 1023u) / 1024u, 1024u>>>(values, mean);
    ref::build_density_grid_bitfield_kernel<<<(ref::NERF_GRID_CELLS / 8u + 127u) / 128u, 128u>>>(values, mean, occupancy, occupied);
    return status_of(cudaDeviceSynchronize());
}

// compute_training_loss_and_compact_kernel (ngp.train.cu:747-860), counters and loss cleared.
int ref_training_loss(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels, uint32_t frame_count,
                      uint32_t width, uint32_t height, const uint16_t* network_output, uint32_t* compacted_counter, const uint32_t* ray_indices,
                      const float* rays, uint32_t* numsteps, const float* coords, float* coords_out, uint16_t* dloss, float* loss) {
    cudaMemset(compacted_counter, 0, 4);
    cudaMemset(loss, 0, sizeof(float) * rays_per_batch);
    ref::compute_training_loss_and_compact_kernel<<<(rays_per_batch + 127u) / 128u, 128u>>>(
        rays_per_batch, step, ray_counter, pixels, frame_count, width, height, reinterpret_cast<const __half*>(network_output), compacted_counter,
        ray_indices, rays, numsteps, coords, coords_out, reinterpret_cast<__half*>(dloss), loss);
    return status_of(cudaDeviceSynchronize());
}

// adam_step_kernel (ngp.train.cu:1261-1280) over the reference's full parameter vector.
int ref_adam(float* master, uint16_t* params, const uint16_t* grads, float* m, float* v, uint32_t* steps) {
    const uint32_t n = cfg::NETWORK_PARAMETER_LAYOUT.total_param_count;
    ref::adam_step_kernel<<<(n + 127u) / 128u, 128u>>>(master, reinterpret_cast<__half*>(params), reinterpret_cast<const __half*>(grads), m, v, steps);
    return status_of(cudaDeviceSynchronize());
}

// accumulate_evaluation_loss_kernel (ngp.train.cu:676-745) with the reference's launch shape
// (ngp.train.cu:1647): adds the tile's squared error to *sse, writes the comparison image when
// given (the caller zeroes sse).
int ref_eval_composite(uint32_t tile_pixels, uint32_t pixel_offset, uint32_t image, uint32_t width, uint32_t height, const uint8_t* pixels,
                       const uint32_t* numsteps, const float* coords, const uint16_t* network_output, double* sse, uint8_t* comparison) {
    ref::accumulate_evaluation_loss_kernel<<<(tile_pixels + ref::THREADS_PER_BLOCK - 1u) / ref::THREADS_PER_BLOCK, ref::THREADS_PER_BLOCK>>>(
        tile_pixels, pixel_offset, image, width, height, pixels, numsteps, coords, reinterpret_cast<const __half*>(network_output), sse, comparison);
    return status_of(cudaDeviceSynchronize());
}

// initialize_mlp_parameters + initialize_grid_parameters (ngp.train.cu:1423-1490) on the
// reference's full parameter vector (total_param_count fp32 master, fp16 params and gradients).
int ref_init_params(float* master, uint16_t* params, uint16_t* grads) {
    try {
        ref::initialize_mlp_parameters(master, params, grads);
        ref::initialize_grid_parameters(master, params, grads);
    } catch (const std::exception&) {
        return 1;
    }
    return status_of(cudaDeviceSynchronize());
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

#include "train_replay.inc"

// ---------------------------------------------------------------------------------------------
// Marching of given rays with the reference's own device helpers (intersect_unit_aabb,
// is_density_grid_occupied, advance_to_next_density_voxel; ngp.train.cu:199-249), in the loop of
// generate_evaluation_samples_kernel (ngp.train.cu:609-666) written the same way, so golden
// marching fixtures can be made for rays given on the host.  One thread per ray, slots by ray
// order: the caller passes per-ray output offsets (max 1024 samples per ray).
// ---------------------------------------------------------------------------------------------
namespace {
__global__ void ref_march_given_rays_kernel(uint32_t n, const float* __restrict__ rays, const uint8_t* __restrict__ occupancy,
                                            uint32_t* __restrict__ numsteps_out, float* __restrict__ coords_out) {
    const uint32_t i = threadIdx.x + blockIdx.x * blockDim.x;
    if (i >= n) return;
    numsteps_out[i] = 0u;
    const float* r                        = rays + static_cast<uint64_t>(i) * 6u;
    const float3 ray_origin               = {r[0], r[1], r[2]};
    const float3 ray_direction_normalized = {r[3], r[4], r[5]};
    float tmin                            = 0.0f;
    if (!ref::intersect_unit_aabb(ray_origin, ray_direction_normalized, tmin)) return;
    constexpr float dt         = ref::MIN_CONE_STEPSIZE;
    const float start_t        = tmin + 0.5f * dt;
    const float3 inv_direction = {1.0f / ray_direction_normalized.x, 1.0f / ray_direction_normalized.y, 1.0f / ray_direction_normalized.z};
    std::uint32_t numsteps     = 0u;
    float t                    = start_t;
    float3 pos                 = {};
    float* out                 = coords_out + static_cast<uint64_t>(i) * ref::NERF_STEPS * 7u;
    const float3 warped_direction = {(ray_direction_normalized.x + 1.0f) * 0.5f, (ray_direction_normalized.y + 1.0f) * 0.5f,
                                     (ray_direction_normalized.z + 1.0f) * 0.5f};
    while (numsteps < ref::NERF_STEPS) {
        pos = {ray_origin.x + ray_direction_normalized.x * t, ray_origin.y + ray_direction_normalized.y * t, ray_origin.z + ray_direction_normalized.z * t};
        if (!ref::unit_aabb_contains(pos)) break;
        if (ref::is_density_grid_occupied(pos, occupancy)) {
            float* coord = out + static_cast<uint64_t>(numsteps) * 7u;
            coord[0] = pos.x, coord[1] = pos.y, coord[2] = pos.z, coord[3] = dt;
            coord[4] = warped_direction.x, coord[5] = warped_direction.y, coord[6] = warped_direction.z;
            ++numsteps;
            t += dt;
        } else {
            t = ref::advance_to_next_density_voxel(t, pos, ray_direction_normalized, inv_direction);
        }
    }
    numsteps_out[i] = numsteps;
}
}  // namespace

extern "C" int ref_march_given_rays(uint32_t n, const float* rays, const uint8_t* occupancy, uint32_t* numsteps, float* coords) {
    ref_march_given_rays_kernel<<<(n + 127u) / 128u, 128u>>>(n, rays, occupancy, numsteps, coords);
    return status_of(cudaDeviceSynchronize());
}
