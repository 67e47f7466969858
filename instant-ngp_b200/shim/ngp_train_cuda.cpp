// Drop-in implementation of the reference's device layer, `namespace ngp::cuda`
// (ngp.train.h:107-161), on top of this library's C ABI (include/ngp_b200.h).
//
// A maintainer of the reference compiles this file in place of ngp.train.cu, against the
// reference's own ngp.train.h (it supplies the declarations and the compile-time configuration
// in ngp::cuda::config), and links libngp_b200.so:
//
//     g++ -std=c++20 -O2 -fPIC -I<reference> -I<this repo>/include -c ngp_train_cuda.cpp
//     ... -L<this repo>/instant-ngp_b200 -lngp_b200 -lcudart
//
// Every function keeps the reference's signature, argument meaning, ownership (allocate_*
// null their outputs first and cudaMalloc; free_device_buffers frees) and error behaviour
// (std::runtime_error on any invalid argument or failed CUDA call).  Work runs on the legacy
// default stream, as the reference's does, so the caller's implicit ordering still holds.
//
// Differences a caller can observe, all within the reference's contract:
//  * the opaque handle returned in place of the cuBLASLt handle is this layer's context (scratch
//    buffers of the library's kernels); destroy_cublaslt frees it;
//  * samples and compacted samples are placed in ray order (deterministic) instead of the
//    order of a global atomic;
//  * parameter gradients are accumulated in fp32 and rounded to the fp16 gradient buffer once;
//  * evaluation marches tiles of 2^16 pixels a segment at a time and stops marching a ray once
//    its transmittance is spent (the same images; allocate_evaluation_buffers sizes its per-ray
//    buffer for the larger tiles); network outputs behind a ray's stopping point are not written.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "ngp.train.h"
#include "ngp_b200.h"

namespace {

namespace cfg = ngp::cuda::config;

constexpr uint32_t kGridCells       = 128u * 128u * 128u;
constexpr uint32_t kSampleFloats    = 7u;
constexpr uint32_t kRayFloats       = 6u;
constexpr uint32_t kEvalTile        = 1u << 18;
// Segmented evaluation (as the library's trainer renders): tiles of 2^16 pixel rays, marched
// 64 samples per ray first (MAX_SAMPLES / tile, so the first segment always fits), then 128, then
// the rest; rays stop being marched once their transmittance is spent.
constexpr uint32_t kSegTile         = 1u << 16;
constexpr uint32_t kLrTableCapacity = 1u << 20;
constexpr uint32_t kLrTableBlock    = 4096u;
constexpr float kLossScale          = 128.0f;
constexpr uint32_t kMlp             = cfg::NETWORK_PARAMETER_LAYOUT.mlp_param_count;
constexpr uint32_t kTotal           = cfg::NETWORK_PARAMETER_LAYOUT.total_param_count;
constexpr uint32_t kGridParams      = cfg::NETWORK_PARAMETER_LAYOUT.grid_param_count;

static_assert(cfg::GRID_OUTPUT_WIDTH == 32u, "the fused MLPs take 32 encoded features");
static_assert(kMlp == 10240u, "the fused MLPs are 32-64-16 / 32-64-64-16 without bias");
static_assert(cfg::NETWORK_OUTPUT_WIDTH == 16u && cfg::MLP_WIDTH == 64u);

[[noreturn]] void raise(const char* what) { throw std::runtime_error{std::string{what} + ": " + ngp_last_error()}; }
void check(int status, const char* what) {
    if (status != NGP_OK) raise(what);
}
void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error{std::string{what} + " failed: " + cudaGetErrorString(e)};
}
template <typename T>
void device_alloc(T*& out, size_t count, const char* what) {
    out = nullptr;
    void* raw = nullptr;
    check_cuda(cudaMalloc(&raw, std::max<size_t>(count, 1) * sizeof(T)), what);
    out = static_cast<T*>(raw);
}

// Scratch of the library's kernels that the reference's signatures have no place for.
struct Context {
    ngp_grid_layout layout{};
    uint32_t* march_scratch = nullptr;  // ngp_march_scratch_words(kEvalTile)
    void* loss_scratch      = nullptr;
    size_t loss_scratch_bytes = 0;
    float* mlp_scratch      = nullptr;
    size_t mlp_scratch_floats = 0;
    float* grid_grad        = nullptr;  // fp32 hash-grid gradient, zero between steps
    float* grid_partial     = nullptr;
    float* eval_rays        = nullptr;  // [kEvalTile][6]
    float* lr_table         = nullptr;
    // segmented evaluation: per-ray state carried between segments, row list of the evaluation
    float* seg_tout         = nullptr;  // [kSegTile]
    float* seg_tstate       = nullptr;  // [kSegTile]
    uint32_t* seg_marched   = nullptr;  // [kSegTile]
    float* seg_state        = nullptr;  // [kSegTile][4]
    uint32_t* seg_lists     = nullptr;  // [2][kSegTile]
    uint32_t* seg_counters  = nullptr;  // [4]
    uint32_t* eval_rows     = nullptr;  // [MAX_SAMPLES]
    uint32_t lr_table_len   = 0;
    uint32_t adam_calls     = 0;
};

Context* g_context = nullptr;

Context* context() {
    if (g_context != nullptr) return g_context;
    auto* c = new Context{};
    try {
        check(ngp_grid_layout_make(cfg::GRID_N_LEVELS, cfg::GRID_FEATURES_PER_LEVEL, cfg::GRID_LOG2_HASHMAP_SIZE, cfg::GRID_BASE_RESOLUTION,
                                   1.0, &c->layout),
              "grid layout");
        if (c->layout.n_params != kGridParams) throw std::runtime_error{"grid layout does not match ngp::cuda::config"};
        for (uint32_t l = 0; l <= cfg::GRID_N_LEVELS; ++l)
            if (c->layout.offsets[l] != cfg::NETWORK_PARAMETER_LAYOUT.grid_offsets[l]) throw std::runtime_error{"grid offsets do not match"};
        const uint32_t max_rays = std::max(kEvalTile, cfg::NETWORK_BATCH_SIZE);
        device_alloc(c->march_scratch, ngp_march_scratch_words(max_rays), "cudaMalloc march scratch");
        c->loss_scratch_bytes = ngp_loss_scratch_bytes(cfg::NETWORK_BATCH_SIZE);
        unsigned char* ls     = nullptr;
        device_alloc(ls, c->loss_scratch_bytes, "cudaMalloc loss scratch");
        c->loss_scratch       = ls;
        c->mlp_scratch_floats = ngp_mlp_backward_scratch_floats();
        device_alloc(c->mlp_scratch, c->mlp_scratch_floats, "cudaMalloc mlp scratch");
        device_alloc(c->grid_grad, kGridParams, "cudaMalloc grid gradient");
        check_cuda(cudaMemset(c->grid_grad, 0, sizeof(float) * kGridParams), "cudaMemset grid gradient");
        device_alloc(c->grid_partial, ngp_density_grid_partials(), "cudaMalloc grid partial sums");
        device_alloc(c->eval_rays, static_cast<size_t>(kEvalTile) * kRayFloats, "cudaMalloc evaluation rays");
        device_alloc(c->lr_table, kLrTableCapacity, "cudaMalloc adam rate table");
        device_alloc(c->seg_tout, kSegTile, "cudaMalloc segment t");
        device_alloc(c->seg_tstate, kSegTile, "cudaMalloc segment ray t");
        device_alloc(c->seg_marched, kSegTile, "cudaMalloc segment ray counts");
        device_alloc(c->seg_state, static_cast<size_t>(kSegTile) * 4u, "cudaMalloc segment ray state");
        device_alloc(c->seg_lists, static_cast<size_t>(kSegTile) * 2u, "cudaMalloc segment lists");
        device_alloc(c->seg_counters, 4, "cudaMalloc segment counters");
        device_alloc(c->eval_rows, cfg::MAX_SAMPLES, "cudaMalloc evaluation rows");
    } catch (...) {
        cudaFree(c->march_scratch), cudaFree(c->loss_scratch), cudaFree(c->mlp_scratch), cudaFree(c->grid_grad), cudaFree(c->grid_partial);
        cudaFree(c->eval_rays), cudaFree(c->lr_table);
        cudaFree(c->seg_tout), cudaFree(c->seg_tstate), cudaFree(c->seg_marched), cudaFree(c->seg_state), cudaFree(c->seg_lists),
            cudaFree(c->seg_counters), cudaFree(c->eval_rows);
        delete c;
        throw;
    }
    g_context = c;
    return c;
}

void destroy_context(Context* c) {
    if (c == nullptr) return;
    cudaFree(c->march_scratch), cudaFree(c->loss_scratch), cudaFree(c->mlp_scratch), cudaFree(c->grid_grad), cudaFree(c->grid_partial);
    cudaFree(c->eval_rays), cudaFree(c->lr_table);
    cudaFree(c->seg_tout), cudaFree(c->seg_tstate), cudaFree(c->seg_marched), cudaFree(c->seg_state), cudaFree(c->seg_lists),
        cudaFree(c->seg_counters), cudaFree(c->eval_rows);
    if (g_context == c) g_context = nullptr;
    delete c;
}

const uint16_t* grid_params(const uint16_t* params) { return params + cfg::NETWORK_PARAMETER_LAYOUT.grid_param_offset; }

// Encoding + both networks for n rows (n a multiple of 128).
void run_network(uint32_t n, const float* coords, const uint16_t* params, uint16_t* encoded, uint16_t* output) {
    Context* c = context();
    check(ngp_encode_grid_forward(&c->layout, n, coords, kSampleFloats, grid_params(params), encoded, n, nullptr), "encode_grid_forward");
    check(ngp_mlp_forward(n, params, encoded, n, coords, kSampleFloats, output, nullptr, nullptr), "mlp_forward");
}

}  // namespace

namespace ngp::cuda {

void free_device_buffers(void** pointers, std::size_t count) noexcept {
    for (std::size_t i = 0; i < count; ++i) {
        if (pointers[i] != nullptr) cudaFree(pointers[i]);
        pointers[i] = nullptr;
    }
}

void destroy_cublaslt(void*& handle) noexcept {
    cudaDeviceSynchronize();
    destroy_context(static_cast<Context*>(handle));
    handle = nullptr;
}

void upload_dataset(const std::uint8_t* pixels, std::size_t pixels_bytes, const float* camera, std::size_t camera_count, const std::uint8_t*& out_pixels,
                    const float*& out_camera) {
    out_pixels = nullptr;
    out_camera = nullptr;
    if (pixels == nullptr || pixels_bytes == 0 || camera == nullptr || camera_count == 0) throw std::runtime_error{"invalid dataset upload input."};
    std::uint8_t* p = nullptr;
    device_alloc(p, pixels_bytes, "cudaMalloc pixels");
    out_pixels = p;
    check_cuda(cudaMemcpy(p, pixels, pixels_bytes, cudaMemcpyHostToDevice), "cudaMemcpy pixels");
    float* cam = nullptr;
    device_alloc(cam, camera_count, "cudaMalloc camera");
    out_camera = cam;
    check_cuda(cudaMemcpy(cam, camera, camera_count * sizeof(float), cudaMemcpyHostToDevice), "cudaMemcpy camera");
}

void allocate_sampler_buffers(float*& out_sample_coords, float*& out_rays, std::uint32_t*& out_ray_indices, std::uint32_t*& out_numsteps,
                              std::uint32_t*& out_ray_counter, std::uint32_t*& out_sample_counter, std::uint8_t*& out_occupancy) {
    out_sample_coords = nullptr, out_rays = nullptr, out_ray_indices = nullptr, out_numsteps = nullptr;
    out_ray_counter = nullptr, out_sample_counter = nullptr, out_occupancy = nullptr;
    device_alloc(out_sample_coords, static_cast<size_t>(cfg::MAX_SAMPLES) * kSampleFloats, "cudaMalloc sampler sample coords");
    device_alloc(out_rays, static_cast<size_t>(cfg::NETWORK_BATCH_SIZE) * kRayFloats, "cudaMalloc sampler rays");
    device_alloc(out_ray_indices, cfg::NETWORK_BATCH_SIZE, "cudaMalloc sampler ray indices");
    device_alloc(out_numsteps, static_cast<size_t>(cfg::NETWORK_BATCH_SIZE) * 2u, "cudaMalloc sampler numsteps");
    device_alloc(out_ray_counter, 1, "cudaMalloc sampler ray counter");
    device_alloc(out_sample_counter, 1, "cudaMalloc sampler sample counter");
    device_alloc(out_occupancy, kGridCells / 8u, "cudaMalloc sampler occupancy");
    check_cuda(cudaMemset(out_occupancy, 0xFF, kGridCells / 8u), "cudaMemset sampler occupancy");
}

void sample_training_batch(const float* camera, std::uint32_t frame_count, std::uint32_t width, std::uint32_t height, float focal_x, float focal_y,
                           float principal_x, float principal_y, std::uint32_t current_step, std::uint32_t rays_per_batch, std::uint32_t sample_limit,
                           const std::uint8_t* occupancy, float* sample_coords, float* rays, std::uint32_t* ray_indices, std::uint32_t* numsteps,
                           std::uint32_t* ray_counter, std::uint32_t* sample_counter) {
    if (sample_limit == 0u || sample_limit > cfg::MAX_SAMPLES || rays_per_batch > cfg::NETWORK_BATCH_SIZE || frame_count == 0u || width == 0u ||
        height == 0u || !(focal_x > 0.0f) || !(focal_y > 0.0f) || !std::isfinite(principal_x) || !std::isfinite(principal_y))
        throw std::runtime_error{"invalid sampler input."};
    if (rays_per_batch == 0u) return;
    check(ngp_march_training_rays(camera, frame_count, width, height, focal_x, focal_y, principal_x, principal_y, current_step, rays_per_batch, nullptr,
                                  sample_limit, occupancy, sample_coords, rays, ray_indices, numsteps, context()->march_scratch, ray_counter,
                                  sample_counter, nullptr),
          "sample_training_batch");
}

void allocate_density_grid_buffers(float*& out_density_grid_values, float*& out_density_grid_scratch, std::uint32_t*& out_density_grid_indices,
                                   float*& out_density_grid_mean, std::uint32_t*& out_density_grid_occupied_count) {
    out_density_grid_values = nullptr, out_density_grid_scratch = nullptr, out_density_grid_indices = nullptr;
    out_density_grid_mean = nullptr, out_density_grid_occupied_count = nullptr;
    device_alloc(out_density_grid_values, kGridCells, "cudaMalloc density grid values");
    device_alloc(out_density_grid_scratch, kGridCells, "cudaMalloc density grid scratch");
    device_alloc(out_density_grid_indices, kGridCells, "cudaMalloc density grid indices");
    device_alloc(out_density_grid_mean, 1, "cudaMalloc density grid mean");
    device_alloc(out_density_grid_occupied_count, 1, "cudaMalloc density grid occupied count");
    check_cuda(cudaMemset(out_density_grid_values, 0, sizeof(float) * kGridCells), "cudaMemset density grid values");
    check_cuda(cudaMemset(out_density_grid_scratch, 0, sizeof(float) * kGridCells), "cudaMemset density grid scratch");
    check_cuda(cudaMemset(out_density_grid_mean, 0, sizeof(float)), "cudaMemset density grid mean");
    check_cuda(cudaMemset(out_density_grid_occupied_count, 0, sizeof(std::uint32_t)), "cudaMemset density grid occupied count");
}

void update_density_grid(const float* camera, std::uint32_t frame_count, std::uint32_t width, std::uint32_t height, float focal_x, float focal_y,
                         float principal_x, float principal_y, std::uint32_t current_step, const std::uint16_t* params, float* sample_coords,
                         std::uint16_t* density_input, std::uint16_t* density_grid_output, float* density_grid_values, float* density_grid_scratch,
                         std::uint32_t* density_grid_indices, float* density_grid_mean, std::uint32_t* density_grid_occupied_count,
                         std::uint8_t* occupancy, std::uint32_t& density_grid_ema_step, float& out_elapsed_ms) {
    out_elapsed_ms = 0.0f;
    uint32_t skip  = current_step / 16u;  // the reference's schedule (ngp.train.cu:1527-1531)
    skip           = std::clamp(skip, 1u, 16u);
    if (current_step % skip != 0u) return;
    if (frame_count == 0u || width == 0u || height == 0u || !(focal_x > 0.0f) || !(focal_y > 0.0f) || !std::isfinite(principal_x) ||
        !std::isfinite(principal_y) || camera == nullptr || params == nullptr || sample_coords == nullptr || density_input == nullptr ||
        density_grid_output == nullptr || density_grid_values == nullptr || density_grid_scratch == nullptr || density_grid_indices == nullptr ||
        density_grid_mean == nullptr || density_grid_occupied_count == nullptr || occupancy == nullptr)
        throw std::runtime_error{"invalid density grid update input."};
    const auto start   = std::chrono::steady_clock::now();
    Context* c         = context();
    const uint32_t n_u = current_step < 256u ? kGridCells : kGridCells / 4u;
    const uint32_t n_n = current_step < 256u ? 0u : kGridCells / 4u;
    if (current_step == 0u) {
        density_grid_ema_step = 0u;
        check(ngp_density_grid_mark_untrained(camera, frame_count, width, height, focal_x, focal_y, principal_x, principal_y, density_grid_values,
                                              nullptr),
              "mark untrained density grid");
    }
    check(ngp_density_grid_samples(n_u, n_n, density_grid_ema_step, density_grid_values, sample_coords, density_grid_indices, nullptr),
          "density grid samples");
    const uint32_t n = n_u + n_n;
    check(ngp_encode_grid_forward(&c->layout, n, sample_coords, kSampleFloats, grid_params(params), density_input, n, nullptr), "density grid encode");
    check(ngp_density_forward(n, params, density_input, n, density_grid_output, nullptr), "density grid mlp");
    check(ngp_density_grid_splat(n, density_grid_indices, density_grid_output, density_grid_scratch, nullptr), "density grid splat");
    check(ngp_density_grid_update(density_grid_values, density_grid_scratch, 0.95f, c->grid_partial, density_grid_mean, occupancy,
                                  density_grid_occupied_count, nullptr),
          "density grid update");
    ++density_grid_ema_step;
    check_cuda(cudaDeviceSynchronize(), "density grid update synchronization");
    out_elapsed_ms = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - start).count();
}

void allocate_training_loss_buffers(std::uint32_t*& out_compacted_sample_counter, float*& out_compacted_sample_coords, float*& out_loss_values) {
    out_compacted_sample_counter = nullptr, out_compacted_sample_coords = nullptr, out_loss_values = nullptr;
    device_alloc(out_compacted_sample_counter, 1, "cudaMalloc compacted sample counter");
    device_alloc(out_compacted_sample_coords, static_cast<size_t>(cfg::NETWORK_BATCH_SIZE) * kSampleFloats, "cudaMalloc compacted sample coords");
    device_alloc(out_loss_values, cfg::NETWORK_BATCH_SIZE, "cudaMalloc loss values");
}

void compute_training_loss_and_compact_samples(std::uint32_t rays_per_batch, std::uint32_t current_step, const std::uint32_t* ray_counter,
                                               const std::uint8_t* pixels, std::uint32_t frame_count, std::uint32_t width, std::uint32_t height,
                                               const std::uint16_t* network_output, std::uint32_t* compacted_sample_counter,
                                               const std::uint32_t* ray_indices, const float* rays, std::uint32_t* numsteps, const float* sample_coords,
                                               float* compacted_sample_coords, std::uint16_t* network_output_gradients, float* loss_values) {
    if (rays_per_batch == 0u) return;
    if (rays_per_batch > cfg::NETWORK_BATCH_SIZE || ray_counter == nullptr) throw std::runtime_error{"invalid loss and compaction input."};
    Context* c = context();
    check(ngp_training_loss_and_compact(rays_per_batch, current_step, ray_counter, pixels, frame_count, width, height, network_output,
                                        compacted_sample_counter, ray_indices, rays, numsteps, sample_coords, compacted_sample_coords,
                                        network_output_gradients, loss_values, c->loss_scratch, c->loss_scratch_bytes, nullptr),
          "compute_training_loss_and_compact_samples");
}

void pad_compacted_training_batch(const std::uint32_t* compacted_sample_counter, float* compacted_sample_coords, std::uint16_t* network_output_gradients) {
    check(ngp_pad_training_batch(compacted_sample_counter, compacted_sample_coords, network_output_gradients, nullptr), "pad_compacted_training_batch");
}

void allocate_evaluation_buffers(std::uint32_t*& out_evaluation_numsteps, std::uint32_t*& out_evaluation_sample_counter,
                                 std::uint32_t*& out_evaluation_overflow_counter, double*& out_evaluation_loss_sum) {
    out_evaluation_numsteps = nullptr, out_evaluation_sample_counter = nullptr, out_evaluation_overflow_counter = nullptr;
    out_evaluation_loss_sum = nullptr;
    device_alloc(out_evaluation_numsteps, static_cast<size_t>(kEvalTile) * 2u, "cudaMalloc evaluation numsteps");
    device_alloc(out_evaluation_sample_counter, 1, "cudaMalloc evaluation sample counter");
    device_alloc(out_evaluation_overflow_counter, 1, "cudaMalloc evaluation overflow counter");
    device_alloc(out_evaluation_loss_sum, 1, "cudaMalloc evaluation loss sum");
}

void allocate_test_comparison_buffer(std::uint32_t width, std::uint32_t height, std::uint8_t*& out_test_comparison_pixels) {
    out_test_comparison_pixels = nullptr;
    if (width == 0u || height == 0u) throw std::runtime_error{"invalid test comparison image dimensions."};
    device_alloc(out_test_comparison_pixels, static_cast<size_t>(width) * height * 2u * 3u, "cudaMalloc test comparison image");
}

void run_evaluation(const std::uint8_t* evaluation_pixels, const float* evaluation_camera, std::uint32_t evaluation_frame_count,
                    std::uint32_t evaluation_image_begin, std::uint32_t evaluation_image_count, std::uint32_t width, std::uint32_t height, float focal_x,
                    float focal_y, float principal_x, float principal_y, const std::uint8_t* occupancy, const std::uint16_t* params, float* sample_coords,
                    std::uint16_t* density_input, std::uint16_t* rgb_input, std::uint16_t* network_output, std::uint32_t* evaluation_numsteps,
                    std::uint32_t* evaluation_sample_counter, std::uint32_t* evaluation_overflow_counter, double* evaluation_loss_sum,
                    std::uint8_t* test_comparison_pixels, std::uint8_t* host_test_comparison_pixels, double& out_loss_sum) {
    out_loss_sum                 = 0.0;
    const bool writes_comparison = test_comparison_pixels != nullptr || host_test_comparison_pixels != nullptr;
    if (evaluation_pixels == nullptr || evaluation_camera == nullptr || evaluation_frame_count == 0u || evaluation_image_count == 0u || width == 0u ||
        height == 0u || !(focal_x > 0.0f) || !(focal_y > 0.0f) || !std::isfinite(principal_x) || !std::isfinite(principal_y) || occupancy == nullptr ||
        params == nullptr || sample_coords == nullptr || density_input == nullptr || rgb_input == nullptr || network_output == nullptr ||
        evaluation_numsteps == nullptr || evaluation_sample_counter == nullptr || evaluation_overflow_counter == nullptr || evaluation_loss_sum == nullptr)
        throw std::runtime_error{"invalid evaluation input."};
    if (evaluation_image_begin >= evaluation_frame_count || evaluation_image_count > evaluation_frame_count - evaluation_image_begin)
        throw std::runtime_error{"evaluation image range is out of bounds."};
    if (writes_comparison && (test_comparison_pixels == nullptr || host_test_comparison_pixels == nullptr || evaluation_image_count != 1u))
        throw std::runtime_error{"test comparison output requires exactly one evaluation image."};
    const uint64_t total64 = static_cast<uint64_t>(width) * height;
    if (total64 > 0xFFFFFFFFull) throw std::runtime_error{"evaluation image has too many pixels."};
    const auto total = static_cast<uint32_t>(total64);
    Context* c       = context();
    check_cuda(cudaMemset(evaluation_loss_sum, 0, sizeof(double)), "cudaMemset evaluation loss sum");
    check_cuda(cudaMemset(evaluation_overflow_counter, 0, sizeof(uint32_t)), "cudaMemset evaluation overflow counter");
    for (uint32_t k = 0; k < evaluation_image_count; ++k) {
        const uint32_t image = evaluation_image_begin + k;
        for (uint32_t offset = 0; offset < total; offset += kSegTile) {
            const uint32_t n = std::min(kSegTile, total - offset);
            check(ngp_make_eval_rays(evaluation_camera, image, width, height, focal_x, focal_y, principal_x, principal_y, offset, n, c->eval_rays, nullptr),
                  "evaluation rays");
            uint32_t max_entries = n;
            for (uint32_t seg = 0;; ++seg) {
                const bool first      = seg == 0;
                const uint32_t* list  = first ? nullptr : c->seg_lists + static_cast<size_t>((seg - 1u) & 1u) * kSegTile;
                const uint32_t* n_dev = first ? nullptr : c->seg_counters + 2u + ((seg - 1u) & 1u);
                const uint32_t cap    = seg == 0 ? cfg::MAX_SAMPLES / kSegTile : (seg == 1 ? 128u : 1024u);
                check(ngp_march_rays_segment(max_entries, n_dev, list, c->eval_rays, occupancy, first ? nullptr : c->seg_tstate,
                                             first ? nullptr : c->seg_marched, cap, cfg::MAX_SAMPLES, sample_coords, evaluation_numsteps, c->seg_tout,
                                             c->march_scratch, c->seg_counters, nullptr),
                      "evaluation march");
                uint32_t h[4] = {};
                check_cuda(cudaMemcpy(h, c->seg_counters, sizeof(h), cudaMemcpyDeviceToHost), "cudaMemcpy evaluation counters");
                const uint32_t complete = h[1];
                if (complete == 0) break;  // no rays left in this tile
                const uint32_t used = std::min(h[0], cfg::MAX_SAMPLES);
                if (used > 0)
                    check(ngp_eval_network_progressive(complete, &c->layout, params, sample_coords, used, evaluation_numsteps, density_input, used,
                                                       network_output, c->eval_rows, c->loss_scratch, c->loss_scratch_bytes, nullptr),
                          "evaluation network");
                uint32_t* next_count = c->seg_counters + 2u + (seg & 1u);
                check_cuda(cudaMemset(next_count, 0, sizeof(uint32_t)), "cudaMemset evaluation list count");
                check(ngp_eval_composite_segment(max_entries, n_dev, c->seg_counters + 1, list, evaluation_numsteps, sample_coords, network_output,
                                                 c->seg_tout, c->seg_tstate, c->seg_marched, c->seg_state,
                                                 c->seg_lists + static_cast<size_t>(seg & 1u) * kSegTile, next_count, offset, image, width, height,
                                                 evaluation_pixels, evaluation_loss_sum, writes_comparison ? test_comparison_pixels : nullptr, nullptr,
                                                 nullptr),
                      "evaluation compositing");
                if (!first) max_entries = h[2u + ((seg - 1u) & 1u)];
            }
        }
    }
    check_cuda(cudaDeviceSynchronize(), "evaluation synchronization");
    check_cuda(cudaMemcpy(&out_loss_sum, evaluation_loss_sum, sizeof(double), cudaMemcpyDeviceToHost), "cudaMemcpy evaluation loss sum");
    if (writes_comparison)
        check_cuda(cudaMemcpy(host_test_comparison_pixels, test_comparison_pixels, total64 * 6u, cudaMemcpyDeviceToHost), "cudaMemcpy test comparison image");
}

void allocate_network_buffers(std::uint16_t*& out_density_input, std::uint16_t*& out_rgb_input, std::uint16_t*& out_network_output,
                              std::uint16_t*& out_network_output_gradients, std::uint16_t*& out_rgb_output_gradients,
                              std::uint16_t*& out_rgb_input_gradients, std::uint16_t*& out_density_input_gradients,
                              std::uint16_t*& out_density_forward_hidden, std::uint16_t*& out_rgb_forward_hidden,
                              std::uint16_t*& out_density_backward_hidden, std::uint16_t*& out_rgb_backward_hidden, void*& out_cublaslt_handle,
                              std::uint8_t*& out_cublaslt_workspace) {
    out_density_input = out_rgb_input = out_network_output = out_network_output_gradients = out_rgb_output_gradients = nullptr;
    out_rgb_input_gradients = out_density_input_gradients = out_density_forward_hidden = out_rgb_forward_hidden = nullptr;
    out_density_backward_hidden = out_rgb_backward_hidden = nullptr;
    out_cublaslt_handle    = nullptr;
    out_cublaslt_workspace = nullptr;
    out_cublaslt_handle    = context();
    // The encodings of every pre-compaction sample are produced at once (no 2^18 chunks), so the
    // network input holds MAX_SAMPLES columns.  The hidden-activation buffers are kept for the
    // signature only: the fused kernels hold activations on chip.
    device_alloc(out_density_input, static_cast<size_t>(cfg::GRID_OUTPUT_WIDTH) * cfg::MAX_SAMPLES, "cudaMalloc density network input");
    device_alloc(out_rgb_input, 16, "cudaMalloc rgb network input");
    device_alloc(out_network_output, static_cast<size_t>(cfg::NETWORK_OUTPUT_WIDTH) * cfg::MAX_SAMPLES, "cudaMalloc network output");
    device_alloc(out_network_output_gradients, static_cast<size_t>(cfg::NETWORK_OUTPUT_WIDTH) * cfg::NETWORK_BATCH_SIZE,
                 "cudaMalloc network output gradients");
    device_alloc(out_rgb_output_gradients, 16, "cudaMalloc rgb output gradients");
    device_alloc(out_rgb_input_gradients, 16, "cudaMalloc rgb input gradients");
    device_alloc(out_density_input_gradients, static_cast<size_t>(cfg::GRID_OUTPUT_WIDTH) * cfg::NETWORK_BATCH_SIZE, "cudaMalloc density input gradients");
    device_alloc(out_density_forward_hidden, 16, "cudaMalloc density forward hidden");
    device_alloc(out_rgb_forward_hidden, 16, "cudaMalloc rgb forward hidden");
    device_alloc(out_density_backward_hidden, 16, "cudaMalloc density backward hidden");
    device_alloc(out_rgb_backward_hidden, 16, "cudaMalloc rgb backward hidden");
    device_alloc(out_cublaslt_workspace, 16, "cudaMalloc workspace");
}

void allocate_trainable_parameter_buffers(float*& out_params_full_precision, std::uint16_t*& out_params, std::uint16_t*& out_param_gradients) {
    out_params_full_precision = nullptr, out_params = nullptr, out_param_gradients = nullptr;
    device_alloc(out_params_full_precision, kTotal, "cudaMalloc trainable params full precision");
    device_alloc(out_params, kTotal, "cudaMalloc trainable params");
    device_alloc(out_param_gradients, kTotal, "cudaMalloc trainable param gradients");
}

void initialize_mlp_parameters(float* params_full_precision, std::uint16_t* params, std::uint16_t* param_gradients) {
    if (params_full_precision == nullptr || params == nullptr || param_gradients == nullptr) throw std::runtime_error{"invalid mlp parameter initialization input."};
    check(ngp_init_mlp_parameters(params_full_precision, params, nullptr), "initialize_mlp_parameters");
    check_cuda(cudaMemset(param_gradients, 0, sizeof(std::uint16_t) * kMlp), "cudaMemset mlp gradients");
}

void initialize_grid_parameters(float* params_full_precision, std::uint16_t* params, std::uint16_t* param_gradients) {
    if (params_full_precision == nullptr || params == nullptr || param_gradients == nullptr) throw std::runtime_error{"grid parameter buffers are null."};
    const uint32_t off = cfg::NETWORK_PARAMETER_LAYOUT.grid_param_offset;
    check(ngp_init_grid_parameters(kGridParams, params_full_precision + off, params + off, nullptr), "initialize_grid_parameters");
    check_cuda(cudaMemset(param_gradients + off, 0, sizeof(std::uint16_t) * kGridParams), "cudaMemset grid gradients");
}

void download_trainable_parameters(const float* params_full_precision, float* out_params_full_precision) {
    if (params_full_precision == nullptr || out_params_full_precision == nullptr) throw std::runtime_error{"invalid trainable parameter download input."};
    check_cuda(cudaMemcpy(out_params_full_precision, params_full_precision, sizeof(float) * kTotal, cudaMemcpyDeviceToHost), "cudaMemcpy trainable params download");
}

void upload_trainable_parameters(const float* params_full_precision, float* out_params_full_precision, std::uint16_t* out_params,
                                 std::uint16_t* out_param_gradients, float* optimizer_first_moments, float* optimizer_second_moments,
                                 std::uint32_t* optimizer_param_steps) {
    if (params_full_precision == nullptr || out_params_full_precision == nullptr || out_params == nullptr || out_param_gradients == nullptr ||
        optimizer_first_moments == nullptr || optimizer_second_moments == nullptr || optimizer_param_steps == nullptr)
        throw std::runtime_error{"invalid trainable parameter upload input."};
    check_cuda(cudaMemcpy(out_params_full_precision, params_full_precision, sizeof(float) * kTotal, cudaMemcpyHostToDevice), "cudaMemcpy trainable params upload");
    check_cuda(cudaMemset(out_param_gradients, 0, sizeof(std::uint16_t) * kTotal), "cudaMemset loaded param gradients");
    check_cuda(cudaMemset(optimizer_first_moments, 0, sizeof(float) * kTotal), "cudaMemset loaded optimizer first moments");
    check_cuda(cudaMemset(optimizer_second_moments, 0, sizeof(float) * kTotal), "cudaMemset loaded optimizer second moments");
    check_cuda(cudaMemset(optimizer_param_steps, 0, sizeof(std::uint32_t) * kTotal), "cudaMemset loaded optimizer param steps");
    check(ngp_cast_to_half(kTotal, out_params_full_precision, out_params, nullptr), "cast params to half");
}

void evaluate_network(std::uint32_t sample_count, const float* sample_coords, const std::uint16_t* params, std::uint16_t* density_input,
                      std::uint16_t* rgb_input, std::uint16_t* network_output) {
    if (sample_count == 0u) return;
    if (sample_count % cfg::NETWORK_BATCH_GRANULARITY != 0u || sample_count > cfg::MAX_SAMPLES || sample_coords == nullptr || params == nullptr ||
        density_input == nullptr || rgb_input == nullptr || network_output == nullptr)
        throw std::runtime_error{"invalid network inference input."};
    run_network(sample_count, sample_coords, params, density_input, network_output);
}

void forward_network(const float* sample_coords, const std::uint16_t* params, std::uint16_t* density_input, std::uint16_t* rgb_input,
                     std::uint16_t* density_forward_hidden, std::uint16_t* rgb_forward_hidden, std::uint16_t* network_output) {
    if (sample_coords == nullptr || params == nullptr || density_input == nullptr || rgb_input == nullptr || density_forward_hidden == nullptr ||
        rgb_forward_hidden == nullptr || network_output == nullptr)
        throw std::runtime_error{"invalid network forward input."};
    // the backward recomputes the hidden activations on chip; it needs only the batch's encodings
    run_network(cfg::NETWORK_BATCH_SIZE, sample_coords, params, density_input, network_output);
}

void backward_network(const float* sample_coords, const std::uint16_t* params, std::uint16_t* gradients, const std::uint16_t* density_input,
                      const std::uint16_t* rgb_input, const std::uint16_t* density_forward_hidden, const std::uint16_t* rgb_forward_hidden,
                      const std::uint16_t* network_output, const std::uint16_t* network_output_gradients, std::uint16_t* rgb_output_gradients,
                      std::uint16_t* rgb_input_gradients, std::uint16_t* density_input_gradients, std::uint16_t* density_backward_hidden,
                      std::uint16_t* rgb_backward_hidden, void* cublaslt_handle, std::uint8_t* cublaslt_workspace) {
    if (sample_coords == nullptr || params == nullptr || gradients == nullptr || density_input == nullptr || network_output_gradients == nullptr ||
        density_input_gradients == nullptr || cublaslt_handle == nullptr)
        throw std::runtime_error{"invalid network backward input."};
    auto* c            = static_cast<Context*>(cublaslt_handle);
    constexpr uint32_t B = cfg::NETWORK_BATCH_SIZE;
    // MLP weight gradients straight into the fp16 gradient buffer; input gradients for the grid
    check(ngp_mlp_backward(B, params, density_input, B, sample_coords, kSampleFloats, network_output_gradients, density_input_gradients, B,
                           c->mlp_scratch, c->mlp_scratch_floats, nullptr, gradients, 1.0f, nullptr),
          "mlp backward");
    // hash-grid gradient accumulated in fp32, rounded once into the fp16 buffer (and cleared)
    check(ngp_encode_grid_backward(&c->layout, B, sample_coords, kSampleFloats, density_input_gradients, B, c->grid_grad, nullptr), "grid backward");
    check(ngp_gradients_to_half(kGridParams, c->grid_grad, gradients + cfg::NETWORK_PARAMETER_LAYOUT.grid_param_offset, 1, nullptr), "grid gradients");
}

void allocate_adam_state(float*& out_first_moments, float*& out_second_moments, std::uint32_t*& out_param_steps) {
    out_first_moments = nullptr, out_second_moments = nullptr, out_param_steps = nullptr;
    device_alloc(out_first_moments, kTotal, "cudaMalloc optimizer first moments");
    device_alloc(out_second_moments, kTotal, "cudaMalloc optimizer second moments");
    device_alloc(out_param_steps, kTotal, "cudaMalloc optimizer param steps");
    check_cuda(cudaMemset(out_first_moments, 0, sizeof(float) * kTotal), "cudaMemset optimizer first moments");
    check_cuda(cudaMemset(out_second_moments, 0, sizeof(float) * kTotal), "cudaMemset optimizer second moments");
    check_cuda(cudaMemset(out_param_steps, 0, sizeof(std::uint32_t) * kTotal), "cudaMemset optimizer param steps");
}

void step_optimizer(float* params_full_precision, std::uint16_t* params, const std::uint16_t* gradients, float* first_moments, float* second_moments,
                    std::uint32_t* param_steps) {
    if (params_full_precision == nullptr || params == nullptr || gradients == nullptr || first_moments == nullptr || second_moments == nullptr ||
        param_steps == nullptr)
        throw std::runtime_error{"invalid optimizer input."};
    Context* c = context();
    if (c->adam_calls + 1u > c->lr_table_len && c->lr_table_len < kLrTableCapacity) {
        const uint32_t first = c->lr_table_len + 1u, count = std::min(kLrTableBlock, kLrTableCapacity - first);
        check(ngp_adam_lr_table(c->lr_table, first, count, 1e-2f, 0.9f, 0.99f, nullptr), "adam rate table");
        c->lr_table_len += count;
    }
    ++c->adam_calls;  // bounds every parameter's step count
    check(ngp_adam_step_f16(kTotal, kMlp, 1e-2f, 0.9f, 0.99f, 1e-15f, 1e-6f, kLossScale, params_full_precision, params, gradients, first_moments,
                            second_moments, param_steps, c->lr_table, c->lr_table_len, nullptr),
          "step_optimizer");
}

void read_counter(const std::uint32_t* counter, std::uint32_t& out_value) {
    if (counter == nullptr) throw std::runtime_error{"counter is null."};
    check_cuda(cudaMemcpy(&out_value, counter, sizeof(std::uint32_t), cudaMemcpyDeviceToHost), "cudaMemcpy counter");
}

void read_loss_sum(const float* loss_values, std::uint32_t loss_count, float& out_loss_sum) {
    out_loss_sum = 0.0f;
    if (loss_count == 0u) return;
    if (loss_values == nullptr) throw std::runtime_error{"loss values are null."};
    std::vector<float> host(loss_count);
    check_cuda(cudaMemcpy(host.data(), loss_values, sizeof(float) * loss_count, cudaMemcpyDeviceToHost), "cudaMemcpy loss values");
    for (const float l : host) out_loss_sum += l;
}

}  // namespace ngp::cuda
