/*
 * ngp_b200.h -- C ABI of the B200-native (sm_100a) NeRF training / rendering hot path.
 *
 * Every entry point takes plain device pointers, sizes and an optional CUDA stream
 * (`void* stream`, NULL = legacy default stream), launches hand-written sm_100a kernels,
 * and returns an `int` status (NGP_OK on success).  On failure a message describing the
 * error is kept per host thread and can be read with ngp_last_error().  Nothing in this
 * header depends on torch, CUDA headers or C++.
 *
 * The functions replace the device layer of the reference's `ngp::cuda` namespace
 * (ngp.train.h:107-161, implemented in ngp.train.cu); each declaration names the reference
 * symbol it stands in for.  The drop-in layer instant-ngp_b200/shim/ngp_train_cuda.cpp defines
 * the reference's exact `ngp::cuda` signatures on top of these functions; it is compiled against
 * the reference's own ngp.train.h (no copy of that header ships here).
 *
 * Data layouts (identical to the reference's, ngp.train.cu:38, 563-570, 917-920, 1241):
 *   sample record      7 x fp32 {x, y, z, dt, (dx+1)/2, (dy+1)/2, (dz+1)/2}, array of structs
 *   encoded features   fp16, feature-major [n_levels * F][stride]
 *   hash-grid table    fp16 [entries][F], levels back to back at layout.offsets[level]
 *   network output     fp16 row-major [n][16]; channels 0-2 raw rgb, channel 3 raw density
 */
#ifndef NGP_B200_H
#define NGP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NGP_API __attribute__((visibility("default")))
#else
#define NGP_API
#endif

#define NGP_OK 0
#define NGP_ERR_INVALID 1   /* bad argument: null pointer, size out of range, bad layout   */
#define NGP_ERR_CUDA 2      /* a CUDA runtime call or kernel launch failed                  */
#define NGP_ERR_OVERFLOW 3  /* a device-side budget overflowed (e.g. evaluation samples)    */
#define NGP_ERR_STATE 4     /* call out of order (e.g. training stopped: no samples)        */
/* Layout flag for the stride argument of encoded-feature buffers (encoding outputs and network
 * inputs): a stride with this bit set means the buffer is row-major [rows][n_levels * F] (the
 * features of one sample contiguous: 64 bytes at the 32-feature configurations) instead of the
 * reference's feature-major [n_levels * F][stride].  With row-major inputs the networks fetch
 * each 64-byte row by asynchronous 16-byte copies.  (The trainer keeps feature-major encodings:
 * the encoding kernel, bound by its gathers' L1 traffic, writes them more cheaply.) */
#define NGP_ROWS 0x80000000u
#define NGP_ERR_TIMEOUT 5   /* a collective did not complete in time; the communicator was aborted */

#define NGP_MAX_LEVELS 32
#define NGP_SAMPLE_FLOATS 7
#define NGP_RAY_FLOATS 6

/* Most recent error message of the calling host thread ("" if none). */
NGP_API const char* ngp_last_error(void);
/* Library version string. */
NGP_API const char* ngp_version(void);

/* Host-side fault injection for testing callers' error paths (no reference counterpart: the
 * reference throws std::runtime_error on a failed CUDA call, ngp.train.cu:1290, and its trainer
 * turns that into std::unexpected, ngp.train.cpp:152-154).  Arms `site` (1 = device allocation of
 * the trainer, 2 = kernel launch, 3 = collective) so that its countdown-th event from now returns
 * NGP_ERR_CUDA with the message "... injected fault (...)"; 0 disarms.  The injected failure is a
 * status returned by the host: no GPU fault is raised.  The environment variable
 * NGP_FAULT_INJECT="alloc:N" | "launch:N" | "collective:N" arms a site when the library loads. */
NGP_API int ngp_fault_inject(int site, int64_t countdown);
/* Kernel launches made by this library in this process so far, all threads and devices
 * (diagnostics for benchmarks; no counterpart in the reference). */
NGP_API uint64_t ngp_kernel_launch_count(void);

/* ------------------------------------------------------------------------------------------
 * Multiresolution hash-grid layout.
 *
 * Level l has scale_l = base * 2^(l * log2_per_level_scale) - 1 (computed in double on the
 * host, stored as float), resolution_l = ceil(scale_l) + 1, and
 * min(roundup8(min(res^3, 2^31-1)), 2^log2_hashmap_size) table entries.  With
 * log2_per_level_scale = 1 this is exactly the reference's integer-doubling layout
 * (ngp.train.h:44-56, ngp.train.cu:885-886); the general scale follows example.py:400-401.
 * ------------------------------------------------------------------------------------------ */
typedef struct ngp_grid_layout {
    uint32_t n_levels;
    uint32_t features_per_level;     /* F: 1, 2, 4 or 8                                   */
    uint32_t log2_hashmap_size;
    uint32_t base_resolution;
    double log2_per_level_scale;
    uint32_t offsets[NGP_MAX_LEVELS + 1]; /* entry offset of each level; [n_levels] = total */
    uint32_t resolution[NGP_MAX_LEVELS];
    float scale[NGP_MAX_LEVELS];
    uint32_t n_entries;              /* offsets[n_levels]                                  */
    uint32_t n_params;               /* n_entries * F                                      */
} ngp_grid_layout;

/* Fill *out.  Replaces config::make_network_parameter_layout (ngp.train.h:44-86, grid part). */
NGP_API int ngp_grid_layout_make(uint32_t n_levels, uint32_t features_per_level, uint32_t log2_hashmap_size,
                         uint32_t base_resolution, double log2_per_level_scale, ngp_grid_layout* out);

/* Forward encoding: out[(l*F + f) * out_stride + i] = trilinear interpolation of level l's
 * 8 corner features at point i.  coords[i * coord_stride + {0,1,2}] in [0,1]^3 (fp32).
 * Accumulation is fp32 (fmaf, corner order 0..7), rounded once to fp16.
 * Replaces encode_grid_forward_kernel (ngp.train.cu:876-921). */
NGP_API int ngp_encode_grid_forward(const ngp_grid_layout* layout, uint32_t n, const float* coords,
                            uint32_t coord_stride, const uint16_t* table, uint16_t* out,
                            uint32_t out_stride, void* stream);

/* Backward encoding: table_grad[e*F + f] += w * dy[(l*F + f) * dy_stride + i] over the 8
 * corners of every point and level, with fp32 vector atomics.  table_grad is fp32 and is
 * accumulated into (zero it first to get the gradient of this batch alone).
 * Replaces encode_grid_backward_kernel (ngp.train.cu:923-960), which accumulates in fp16. */
/* Backward for a batch given as a row list: point r's record is coords[rows[r]], its gradient
 * column r of dy. */
NGP_API int ngp_encode_grid_backward_rows(const ngp_grid_layout* layout, uint32_t n, const uint32_t* rows, const float* coords,
                                          uint32_t coord_stride, const uint16_t* dy, uint32_t dy_stride, float* table_grad, void* stream);

/* Forward for a list of points: point rows[r] for r < min(*n_rows, max_rows) (n_rows may be NULL:
 * max_rows points), read from coords[rows[r]] and written to column rows[r] of out (so out_stride
 * must exceed every listed index).  Used to encode only the samples whose density is needed. */
NGP_API int ngp_encode_grid_forward_rows(const ngp_grid_layout* layout, uint32_t max_rows, const uint32_t* rows, const uint32_t* n_rows,
                                         const float* coords, uint32_t coord_stride, const uint16_t* table, uint16_t* out, uint32_t out_stride,
                                         void* stream);

NGP_API int ngp_encode_grid_backward(const ngp_grid_layout* layout, uint32_t n, const float* coords,
                             uint32_t coord_stride, const uint16_t* dy, uint32_t dy_stride,
                             float* table_grad, void* stream);

/* ------------------------------------------------------------------------------------------
 * Fully fused MLPs (tcgen05 tensor cores, fp32 accumulation in TMEM).
 *
 * params: the 10,240 packed fp16 MLP weights [out][in] in the reference order
 * (ngp.train.h:58-78): density W_in 64x32, density W_out 16x64, rgb W_in 64x32, rgb W_h 64x64,
 * rgb W_out 16x64.  x: encoded positions, fp16 feature-major [32][x_stride].  coords: sample
 * records (the view direction is read from floats 4..6).
 * ------------------------------------------------------------------------------------------ */

/* Degree-4 spherical-harmonics encoding of the view directions -> fp16 [16][out_stride].
 * Replaces encode_spherical_harmonics_kernel (ngp.train.cu:962-993). */
NGP_API int ngp_sh_encode(uint32_t n, const float* coords, uint32_t coord_stride, uint16_t* out, uint32_t out_stride, void* stream);

/* Density + colour network forward for n rows -> out fp16 [n][16] (ch 0-2 raw rgb, ch 3 raw
 * density, as network_output in the reference).  density_rgb_in (optional, may be NULL)
 * receives the 16 density outputs feature-major [16][x_stride], the reference's rgb_input[0..15].
 * Replaces evaluate_network / forward_network (ngp.train.cu:1494-1524, 1660-1684): WMMA
 * kernels K19 and the glue kernels K16, K21. */
NGP_API int ngp_mlp_forward(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const float* coords,
                    uint32_t coord_stride, uint16_t* out, uint16_t* density_rgb_in, void* stream);

/* Density network only -> out[n] = raw density (fp16).  Replaces the density-only
 * mlp_forward_64_relu_kernel launch of update_density_grid (ngp.train.cu:1573). */
NGP_API int ngp_density_forward(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, uint16_t* out, void* stream);
/* Density network with the density-grid splat in its epilogue: for each row i, the raw density d
 * (rounded to fp16 as ngp_density_forward writes it) gives scratch[indices[i]] =
 * max(scratch[indices[i]], exp(d) * sqrt(3)/1024) -- ngp_density_forward followed by
 * ngp_density_grid_splat, bit for bit, without the density array.  Replaces the update's
 * mlp_forward_64_relu_kernel launch and splat_kernel (ngp.train.cu:1573, 426-432). */
NGP_API int ngp_density_forward_splat(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const uint32_t* indices,
                                      float* scratch, void* stream);

/* Full network for a list of rows: input column rows[r] of x and record rows[r] of coords, output
 * row out[rows[r]][16], for r < min(*n_rows, max_rows) (n_rows may be NULL). */
NGP_API int ngp_mlp_forward_rows(uint32_t max_rows, const uint32_t* rows, const uint32_t* n_rows, const uint16_t* params, const uint16_t* x,
                                 uint32_t x_stride, const float* coords, uint32_t coord_stride, uint16_t* out, void* stream);

/* Density network for a list of rows: input column rows[r] of x, output out[rows[r]], for
 * r < min(*n_rows, max_rows) (n_rows may be NULL). */
NGP_API int ngp_density_forward_rows(uint32_t max_rows, const uint32_t* rows, const uint32_t* n_rows, const uint16_t* params, const uint16_t* x,
                                     uint32_t x_stride, uint16_t* out, void* stream);

/* Number of fp32 scratch values ngp_mlp_backward needs (one weight-gradient partial per CTA). */
NGP_API uint32_t ngp_mlp_backward_scratch_floats(void);

/* Network backward for n rows: dy fp16 [n][16] (ch 0-2 rgb, ch 3 density gradient) ->
 * dx fp16 [32][dx_stride] (gradient w.r.t. x; may be NULL) and the weight gradient
 * dw = dw_scale * dL/dW written as fp32 (dw_f32) and/or fp16 (dw_f16) [10240] (either may be
 * NULL).  The forward activations are recomputed on chip.  scratch: caller-allocated device
 * buffer of at least ngp_mlp_backward_scratch_floats() floats.  The weight gradient is summed
 * in a fixed order, so results are deterministic.
 * Replaces backward_network (ngp.train.cu:1686-1895): WMMA kernel K20, cuBLASLt G1-G7 and the
 * glue kernels K22, K23. */
NGP_API int ngp_mlp_backward(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const float* coords,
                     uint32_t coord_stride, const uint16_t* dy, uint16_t* dx, uint32_t dx_stride, float* scratch,
                     size_t scratch_floats, float* dw_f32, uint16_t* dw_f16, float dw_scale, void* stream);

/* ngp_mlp_backward for a batch given as a row list: batch row r reads the features (column
 * rows[r] of x) and record (rows[r] of coords) of sample rows[r]; dy and dx are batch-indexed. */
NGP_API int ngp_mlp_backward_rows(uint32_t n, const uint32_t* rows, const uint16_t* params, const uint16_t* x, uint32_t x_stride,
                                  const float* coords, uint32_t coord_stride, const uint16_t* dy, uint16_t* dx, uint32_t dx_stride,
                                  float* scratch, size_t scratch_floats, float* dw_f32, uint16_t* dw_f16, float dw_scale, void* stream);

/* Sticky device status of the MLP kernels: bit 0 = a tensor-core completion wait timed out.
 * reset != 0 clears it. */
NGP_API int ngp_mlp_status(uint32_t* out_status, int reset);

/* ------------------------------------------------------------------------------------------
 * Occupancy density grid: 128^3 cells in Morton order over the unit cube, fp32 values,
 * uint8 bitfield (8 cells per byte).  camera: 12 floats per frame (three axis columns, then
 * the origin), as built by the reference's dataset loader (ngp.dataset.cpp:47-65).
 * ------------------------------------------------------------------------------------------ */

/* values[c] = 0 if any corner of cell c is seen by some training view, else -1.
 * Replaces mark_untrained_density_grid_kernel (ngp.train.cu:310-381). */
NGP_API int ngp_density_grid_mark_untrained(const float* camera, uint32_t frame_count, uint32_t width, uint32_t height, float focal_x,
                                            float focal_y, float principal_x, float principal_y, float* values, void* stream);

/* n_uniform uniformly chosen cells followed by n_nonuniform cells above the occupancy threshold
 * (up to 10 hashed tries), jittered positions from PCG32(1337) at ema_step -> 7-float records
 * and cell indices.  Replaces generate_density_grid_samples_kernel (ngp.train.cu:383-424). */
NGP_API int ngp_density_grid_samples(uint32_t n_uniform, uint32_t n_nonuniform, uint32_t ema_step, const float* values, float* coords,
                                     uint32_t* indices, void* stream);
/* The same samples as ngp_density_grid_samples (identical records and cell indices), placed in
 * Morton cell order of each sample's first hashed cell instead of sample order, so that the
 * encoding of the samples reads neighbouring table entries across a warp.  Each set holds at
 * most 2^21 samples.  counter: one device word of scratch (unused when n_uniform = 2^21 and
 * n_nonuniform = 0); the order within a warp is fixed, the order of warps is not.  The density
 * grid update consumes the samples with an order-independent atomic max, so its result is the
 * reference's (generate_density_grid_samples_kernel, ngp.train.cu:383-424). */
NGP_API int ngp_density_grid_samples_cell_order(uint32_t n_uniform, uint32_t n_nonuniform, uint32_t ema_step, const float* values, float* coords,
                                                uint32_t* indices, uint32_t* counter, void* stream);
/* The warm-up update's samples (n_uniform = 2^21, n_nonuniform = 0: the first 256 steps) generated
 * and encoded in one pass: out[f][i] (feature-major, out_stride >= 2^21) = the hash-grid encoding of
 * sample i of ngp_density_grid_samples_cell_order(2^21, 0, ema_step, ...) and indices[i] its cell
 * index; the positions are not written.  Equal, bit for bit, to that call followed by
 * ngp_encode_grid_forward on its records.  Replaces generate_density_grid_samples_kernel plus the
 * update's encoding (ngp.train.cu:383-424, 876-921). */
NGP_API int ngp_density_grid_encode_samples(const ngp_grid_layout* layout, uint32_t ema_step, const float* values, const uint16_t* table,
                                            uint16_t* out, uint32_t out_stride, uint32_t* indices, void* stream);

/* scratch[indices[i]] = max(scratch[indices[i]], exp(density[i]) * sqrt(3)/1024).
 * Replaces splat_density_grid_samples_kernel (ngp.train.cu:426-432). */
NGP_API int ngp_density_grid_splat(uint32_t n, const uint32_t* indices, const uint16_t* density, float* scratch, void* stream);


/* Size (floats) of the `partial` buffer of ngp_density_grid_update. */
NGP_API uint32_t ngp_density_grid_partials(void);

/* EMA (values = v < 0 ? v : max(decay * v, scratch)), mean of max(v, 0) in a fixed order
 * (deterministic), bitfield = v > min(0.01, mean), occupied-cell count; clears scratch.
 * Replaces K4-K6 (ngp.train.cu:434-474) and the memsets of update_density_grid. */
NGP_API int ngp_density_grid_update(float* values, float* scratch, float decay, float* partial, float* mean, uint8_t* bitfield,
                                    uint32_t* occupied_count, void* stream);

/* ------------------------------------------------------------------------------------------
 * Ray marching (dt = sqrt(3)/1024, <= 1024 occupied steps, empty-space skipping).  Samples are
 * placed in ray order: numsteps[2i] = samples of ray i, numsteps[2i+1] = its first sample.
 * scratch: ngp_march_scratch_words(n_rays) uint32 of device memory, 8-byte aligned (per-CTA
 * sample totals and each ray's runs of occupied steps, so that samples are written without
 * marching the ray a second time).
 * ------------------------------------------------------------------------------------------ */
NGP_API uint64_t ngp_march_scratch_words(uint32_t max_rays);

/* Training rays of `step` from the cameras (PCG32 pixels, start jitter) -> 7-float sample
 * records, rays [i][6] (origin, unnormalised direction), ray_indices (identity), numsteps,
 * *ray_counter = rays, *sample_counter = samples before the limit.  rays_per_batch_dev
 * (optional) overrides the ray count from device memory (<= rays_per_batch).
 * Replaces generate_training_samples_kernel / sample_training_batch (ngp.train.cu:476-578,
 * 1919-1930). */
NGP_API int ngp_march_training_rays(const float* camera, uint32_t frame_count, uint32_t width, uint32_t height, float focal_x,
                                    float focal_y, float principal_x, float principal_y, uint32_t step, uint32_t rays_per_batch,
                                    const uint32_t* rays_per_batch_dev, uint32_t sample_limit, const uint8_t* bitfield, float* coords,
                                    float* rays, uint32_t* ray_indices, uint32_t* numsteps, uint32_t* scratch, uint32_t* ray_counter,
                                    uint32_t* sample_counter, void* stream);

/* Explicit rays [n][6] (origin, unit direction) in the unit-cube frame; jitter != 0 starts at
 * tmin + U*dt with U the third draw of the training PCG32 stream of ray i at `step` (as
 * training rays do), else at tmin + dt/2 (the evaluation rule, ngp.train.cu:613). */
NGP_API int ngp_march_rays(uint32_t n_rays, const float* rays, int jitter, uint32_t step, const uint8_t* bitfield, uint32_t sample_limit,
                           float* coords, uint32_t* numsteps, uint32_t* scratch, uint32_t* sample_counter, void* stream);

/* Segmented marching of evaluation rays: the reference marches every occupied step of a pixel
 * ray (up to 1024) before compositing, although compositing stops once the transmittance falls
 * below 1e-4.  This marches at most `cap` further samples of each listed ray (list NULL: entry k
 * is ray k of `rays`), continuing each ray where the previous segment stopped, so a ray that
 * stops early is never marched past its first segment; the samples of a ray over all its
 * segments are those of ngp_march_rays (jitter 0), bit for bit.
 *   max_entries / n_entries: entry count (n_entries, optional, on the device, <= max_entries);
 *   t_state, marched: per ray, where it continues and how many samples it has had (both NULL for
 *     the first segment, which must fit: cap * max_entries <= sample_limit);
 *   numsteps[2k], numsteps[2k+1]: entry k's samples in this segment and their first record;
 *   t_out[k]: where entry k's ray continues, -1 if its march has ended;
 *   counters[0] = the segment's samples before the limit, counters[1] = entries [0, n) that fit
 *     under sample_limit (a prefix; the rest were not marched and have numsteps 0);
 *   scratch: ngp_march_scratch_words(max_entries) words.
 * Replaces generate_evaluation_samples_kernel (ngp.train.cu:580-667) in the render loop. */
NGP_API int ngp_march_rays_segment(uint32_t max_entries, const uint32_t* n_entries, const uint32_t* list, const float* rays,
                                   const uint8_t* bitfield, const float* t_state, const uint32_t* marched, uint32_t cap, uint32_t sample_limit,
                                   float* coords, uint32_t* numsteps, float* t_out, uint32_t* scratch, uint32_t* counters, void* stream);

/* Pixel rays [n][6] (origin, unit direction) of pixels [pixel_offset, pixel_offset + n) of image
 * `image`.  Replaces the ray set-up of generate_evaluation_samples_kernel (ngp.train.cu:587-614). */
NGP_API int ngp_make_eval_rays(const float* camera, uint32_t image, uint32_t width, uint32_t height, float focal_x, float focal_y,
                               float principal_x, float principal_y, uint32_t pixel_offset, uint32_t n, float* rays, void* stream);
/* Evaluation rays of slots [slot_offset, slot_offset + n) of a tile set: slot j is pixel
 * (j % 4096) (row-major inside the tile) of the set's tile j / 4096, the set being 64 x 64 tiles
 * first_tile, first_tile + tile_stride, ... of the row-major tile grid.  Slots outside the image
 * get a ray that marches no samples. */
NGP_API int ngp_make_eval_rays_tiles(const float* camera, uint32_t image, uint32_t width, uint32_t height, float focal_x, float focal_y,
                                     float principal_x, float principal_y, uint32_t first_tile, uint32_t tile_stride, uint32_t slot_offset, uint32_t n,
                                     float* rays, void* stream);

/* ------------------------------------------------------------------------------------------
 * Compositing, loss and compaction (batch = 2^18 samples).
 * ------------------------------------------------------------------------------------------ */
NGP_API uint32_t ngp_loss_scratch_bytes(uint32_t max_rays); /* 0 (error set) when the size exceeds 32 bits */

/* Front-to-back compositing with early stop at transmittance < 1e-4, random background, L2
 * loss, analytic compositing backward -> dloss_doutput fp16 [2^18][16] (scaled by
 * 128 / rays_per_batch), compacted samples in ray order, loss_values[ray], numsteps rewritten
 * to the compacted (count, base), *compacted_counter.  scratch: ngp_loss_scratch_bytes bytes,
 * 16-byte aligned.  Replaces compute_training_loss_and_compact_kernel (ngp.train.cu:747-860,
 * 1932-1944). */
NGP_API int ngp_training_loss_and_compact(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels,
                                          uint32_t frame_count, uint32_t width, uint32_t height, const uint16_t* network_output,
                                          uint32_t* compacted_counter, const uint32_t* ray_indices, const float* rays, uint32_t* numsteps,
                                          const float* coords, float* compacted_coords, uint16_t* dloss_doutput, float* loss_values,
                                          void* scratch, size_t scratch_bytes, void* stream);

/* ngp_training_loss_and_compact without any device allocation by the caller or the library.
 * No counterpart in the reference.  For callers that cannot allocate device memory when the loss
 * runs (host callbacks and driver-managed regions where cudaMalloc is not allowed, plugin hosts
 * that give a fixed memory budget): the scratch comes from one static device array of about
 * 5 MiB that each GPU loading the library keeps until the process exits.  Limit: rays_per_batch
 * <= ngp_training_loss_and_compact_noalloc_max_rays() (2^18); larger requests fail with
 * NGP_ERR_INVALID.  The first call on a device looks up the array's device address (with that
 * device current) and should come before any stream capture; the address is kept per device and
 * context, so after a device reset (or a new primary context) the next call looks it up again
 * and should also come before any capture.  All calls on a device share the array: calls whose
 * work overlaps on the GPU race with each other.  The scratch needs no clearing between calls
 * (every byte read is written earlier in the same call). */
NGP_API uint32_t ngp_training_loss_and_compact_noalloc_max_rays(void);
NGP_API int ngp_training_loss_and_compact_noalloc(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels,
                                                  uint32_t frame_count, uint32_t width, uint32_t height, const uint16_t* network_output,
                                                  uint32_t* compacted_counter, const uint32_t* ray_indices, const float* rays, uint32_t* numsteps,
                                                  const float* coords, float* compacted_coords, uint16_t* dloss_doutput, float* loss_values,
                                                  void* stream);

/* Density-first variant of ngp_training_loss_and_compact, used by the trainer: which samples a
 * ray keeps depends only on the densities, so the pre-compaction pass needs only the density
 * network and the colour network runs on the kept samples alone.  Same kept set, order, losses
 * and gradients as ngp_training_loss_and_compact (bit for bit).
 *
 * Rows of the compacted buffers: ngp_compacted_rows() = 2^18 + 1024 (the ray that straddles the
 * batch end is compacted whole, so that its colour can be composited).
 *
 * Step 1: density fp16 [samples] (raw, e.g. from ngp_density_forward) -> compacted records
 * [rows][7], optionally the encoded positions of the kept samples (enc [32][enc_stride] ->
 * compacted_enc [32][rows]), numsteps rewritten to (kept, compacted base), *compacted_counter
 * = min(kept total, 2^18).  scratch: ngp_loss_scratch_bytes(rays_per_batch), 16-byte aligned,
 * passed unchanged to step 2. */
NGP_API uint32_t ngp_compacted_rows(void);
NGP_API int ngp_training_compact_by_density(uint32_t rays_per_batch, const uint32_t* ray_counter, const uint16_t* density, const float* coords,
                                            const uint16_t* enc, uint32_t enc_stride, uint32_t* numsteps, float* compacted_coords,
                                            uint16_t* compacted_enc, uint32_t* compacted_counter, void* scratch, size_t scratch_bytes,
                                            void* stream);

/* Step 1 with the densities evaluated progressively (replaces the encoding + density network
 * over all pre-compaction samples and ngp_training_compact_by_density): a ray keeps its samples
 * up to the first whose transmittance falls below 1e-4, so the samples behind it need no density.
 * Densities are computed for the first 48 samples of every ray, then for the remaining samples of
 * the rays that have not stopped; every evaluated density equals the full pass's value, so the
 * kept counts and the compacted outputs are the same.  params: packed fp16 [MLP | grid];
 * sample_bound: the marched sample count's upper bound (the march's sample limit); enc
 * ([32][enc_stride], enc_stride >= sample_bound), density ([sample_bound]) and rows
 * ([sample_bound] uint32) are caller scratch; only evaluated samples' entries are written.
 * Outputs as ngp_training_compact_by_density; scratch: ngp_loss_scratch_bytes(rays_per_batch). */
NGP_API int ngp_training_compact_progressive(uint32_t rays_per_batch, const uint32_t* ray_counter, const ngp_grid_layout* layout,
                                             const uint16_t* params, const float* coords, uint32_t sample_bound, uint32_t* numsteps,
                                             uint16_t* enc, uint32_t enc_stride, uint16_t* density, uint32_t* rows, float* compacted_coords,
                                             uint16_t* compacted_enc, uint32_t* compacted_counter, void* scratch, size_t scratch_bytes,
                                             void* stream);

/* Selection variant used by the trainer: the progressive rounds, then instead of copying the kept
 * samples, the batch is a row list: batch_rows[cbase + j] = (sample index of) ray i's kept sample j,
 * for every ray whose compacted base cbase lies in the batch (the straddling ray whole; batch_rows
 * holds ngp_compacted_rows() entries), *n_selected = rows listed, *compacted_counter = min(kept
 * total, 2^18), numsteps = (kept, cbase).  The network then runs on the listed rows in place
 * (ngp_mlp_forward_rows), ngp_training_loss_selected composites from the samples' own positions,
 * ngp_pad_training_rows pads the list, and the backward reads the list (ngp_mlp_backward_rows,
 * ngp_encode_grid_backward_rows).  Identical values to the copying flow; no sample data is moved. */
NGP_API int ngp_training_select_progressive(uint32_t rays_per_batch, const uint32_t* ray_counter, const ngp_grid_layout* layout,
                                            const uint16_t* params, const float* coords, uint32_t sample_bound, uint32_t* numsteps,
                                            uint16_t* enc, uint32_t enc_stride, uint16_t* density, uint32_t* rows, uint32_t* batch_rows,
                                            uint32_t* n_selected, uint32_t* compacted_counter, void* scratch, size_t scratch_bytes, void* stream);
/* The same with the first round's window chosen by the caller: round 0 evaluates the first
 * first_window samples of every ray (ngp_training_select_progressive: 48), round 1 the rest of the
 * rays still going; first_window = 0xFFFFFFFF evaluates every sample in one round.  The results
 * do not depend on the window (each sample's density is the same value whichever round computes
 * it); only the work does.  still_active (optional device word, cleared by the call): the number
 * of rays still going after round 0, for choosing the next call's window. */
NGP_API int ngp_training_select_progressive_window(uint32_t rays_per_batch, const uint32_t* ray_counter, const ngp_grid_layout* layout,
                                                   const uint16_t* params, const float* coords, uint32_t sample_bound, uint32_t* numsteps,
                                                   uint16_t* enc, uint32_t enc_stride, uint16_t* density, uint32_t* rows, uint32_t* batch_rows,
                                                   uint32_t* n_selected, uint32_t* compacted_counter, void* scratch, size_t scratch_bytes,
                                                   uint32_t first_window, uint32_t* still_active, void* stream);
/* ngp_training_loss_compacted for the selection flow: network_output [samples][16] and coords
 * are indexed by sample (the kept samples' own positions); dloss_doutput by batch row.  scratch:
 * the one given to ngp_training_select_progressive. */
NGP_API int ngp_training_loss_selected(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels,
                                       uint32_t frame_count, uint32_t width, uint32_t height, const uint16_t* network_output,
                                       const uint32_t* ray_indices, const float* rays, uint32_t* numsteps, const float* coords,
                                       uint16_t* dloss_doutput, float* loss_values, const void* scratch, size_t scratch_bytes, void* stream);
/* ngp_training_loss_selected with a choice of loss (no reference counterpart; the reference's L2
 * is at ngp.train.cu:817-820): loss_kind 0 = L2 (the reference's), 1 = Huber (delta 0.1, divided
 * by 5 so that it equals the L2 loss for residuals |d| <= 0.1: loss d^2 there, 0.2 |d| - 0.01
 * beyond, gradient 2 d there, 0.2 sign(d) beyond). */
NGP_API int ngp_training_loss_selected_kind(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels,
                                            uint32_t frame_count, uint32_t width, uint32_t height, const uint16_t* network_output,
                                            const uint32_t* ray_indices, const float* rays, uint32_t* numsteps, const float* coords,
                                            uint16_t* dloss_doutput, float* loss_values, const void* scratch, size_t scratch_bytes, int loss_kind,
                                            void* stream);
/* Padding of the selected batch to 2^18 rows (rows and gradients, as ngp_pad_training_batch). */
NGP_API int ngp_pad_training_rows(const uint32_t* compacted_counter, uint32_t* batch_rows, uint16_t* dloss_doutput, void* stream);

/* Evaluation (rendering) counterpart: the full network's outputs ([samples][16]) for every
 * sample in front of its ray's stopping point (transmittance < 1e-4, where the evaluation
 * compositing of run_evaluation stops; ngp.train.cu:676-745), evaluated in the same two rounds;
 * outputs behind the stopping points are not written (compositing never reads them).  n_rays rays
 * marched into numsteps/coords (ngp_march_rays); enc [32][enc_stride] and rows [sample_bound]
 * are scratch; scratch: ngp_loss_scratch_bytes(n_rays). */
NGP_API int ngp_eval_network_progressive(uint32_t n_rays, const ngp_grid_layout* layout, const uint16_t* params, const float* coords,
                                         uint32_t sample_bound, const uint32_t* numsteps, uint16_t* enc, uint32_t enc_stride, uint16_t* network_output,
                                         uint32_t* rows, void* scratch, size_t scratch_bytes, void* stream);

/* Step 2, after the full network ran on the compacted rows (compacted_output fp16 [rows][16]):
 * compositing, loss and gradients as ngp_training_loss_and_compact; numsteps ends as
 * (samples in the batch, compacted base). */
NGP_API int ngp_training_loss_compacted(uint32_t rays_per_batch, uint32_t step, const uint32_t* ray_counter, const uint8_t* pixels,
                                        uint32_t frame_count, uint32_t width, uint32_t height, const uint16_t* compacted_output,
                                        const uint32_t* ray_indices, const float* rays, uint32_t* numsteps, const float* compacted_coords,
                                        uint16_t* dloss_doutput, float* loss_values, const void* scratch, size_t scratch_bytes, void* stream);

/* ngp_pad_training_batch that also pads the compacted encoded positions (enc [32][enc_stride]),
 * so that they equal the encoding of the padded records. */
NGP_API int ngp_pad_training_batch_enc(const uint32_t* compacted_counter, float* compacted_coords, uint16_t* dloss_doutput, uint16_t* enc,
                                       uint32_t enc_stride, void* stream);

/* Wrap-around padding of the compacted batch to 2^18 samples, copied gradients scaled by
 * count / 2^18.  Replaces K12/K13 (ngp.train.cu:862-874, 1946-1956). */
NGP_API int ngp_pad_training_batch(const uint32_t* compacted_counter, float* compacted_coords, uint16_t* dloss_doutput, void* stream);

/* Compositing of one segment of a segmented march (ngp_march_rays_segment, same list, numsteps,
 * t_out and counters + 1 as `complete`): each marched entry continues its ray's state
 * (state [ray][4] = T, r, g, b, 16-byte aligned; t_state; marched) over the segment's network
 * outputs.  A ray whose transmittance fell below 1e-4 or whose march ended writes its pixel
 * (pixel_offset + ray) exactly as ngp_eval_composite does; the other rays, and the entries past
 * the segment's sample limit, are appended to next_list (*next_count, cleared by the caller) in
 * no fixed order.  The first segment (list NULL) starts every ray at T = 1.
 * Replaces accumulate_evaluation_loss_kernel (ngp.train.cu:676-745) in the render loop. */
NGP_API int ngp_eval_composite_segment(uint32_t max_entries, const uint32_t* n_entries, const uint32_t* complete, const uint32_t* list,
                                       const uint32_t* numsteps, const float* coords, const uint16_t* network_output, const float* t_out,
                                       float* t_state, uint32_t* marched, float* state, uint32_t* next_list, uint32_t* next_count,
                                       uint32_t pixel_offset, uint32_t image, uint32_t width, uint32_t height, const uint8_t* pixels, double* sse,
                                       uint8_t* comparison, float* rendered, void* stream);
/* ngp_eval_composite_segment whose rays are the slots of a tile set (as ngp_make_eval_rays_tiles;
 * pixel_offset is the slot offset; first_tile = 0xFFFFFFFF: every pixel, row-major). */
NGP_API int ngp_eval_composite_segment_tiles(uint32_t max_entries, const uint32_t* n_entries, const uint32_t* complete, const uint32_t* list,
                                             const uint32_t* numsteps, const float* coords, const uint16_t* network_output, const float* t_out,
                                             float* t_state, uint32_t* marched, float* state, uint32_t* next_list, uint32_t* next_count,
                                             uint32_t pixel_offset, uint32_t image, uint32_t width, uint32_t height, const uint8_t* pixels,
                                             double* sse, uint8_t* comparison, float* rendered, uint32_t first_tile, uint32_t tile_stride,
                                             void* stream);

/* Evaluation compositing of n_pixels pixels: *sse += squared error vs the sRGB target (fp64; no
 * target when pixels is NULL), optional comparison image [height][2*width][3] (target | render)
 * and rendered [pixel][3].  Replaces accumulate_evaluation_loss_kernel (ngp.train.cu:676-745). */
NGP_API int ngp_eval_composite(uint32_t n_pixels, uint32_t pixel_offset, uint32_t image, uint32_t width, uint32_t height, const uint8_t* pixels,
                               const uint32_t* numsteps, const float* coords, const uint16_t* network_output, double* sse,
                               uint8_t* comparison, float* rendered, void* stream);

/* ------------------------------------------------------------------------------------------
 * Optimizer.  Parameters [0, n_mlp) dense with L2 regularisation, the rest sparse (zero
 * gradient = skipped).  gradients are fp32 and divided by loss_scale; clear_grid_gradients != 0
 * zeroes gradients [n_mlp, n_params) in the same pass.  n_mlp % 4 == 0.
 * Replaces adam_step_kernel / step_optimizer (ngp.train.cu:1261-1280, 1973-1980).
 * ------------------------------------------------------------------------------------------ */
NGP_API int ngp_adam_step(uint32_t n_params, uint32_t n_mlp, float lr, float beta1, float beta2, float eps, float l2_reg, float loss_scale,
                          float* params_full_precision, uint16_t* params, float* gradients, float* first_moments, float* second_moments,
                          uint32_t* param_steps, int clear_grid_gradients, void* stream);

/* The bias-corrected rate lr * sqrt(1 - beta2^t) / (1 - beta1^t) for t in [first, first + count)
 * -> table[t].  With such a table, ngp_adam_step_table reads the rate of each parameter's step
 * count instead of evaluating two powf per parameter (same values: the same function of t). */
NGP_API int ngp_adam_lr_table(float* table, uint32_t first, uint32_t count, float lr, float beta1, float beta2, void* stream);

/* ngp_adam_step using lr_table[1 .. table_len] (filled by ngp_adam_lr_table with the same lr and
 * betas); step counts beyond table_len fall back to computing the rate. */
NGP_API int ngp_adam_step_table(uint32_t n_params, uint32_t n_mlp, float lr, float beta1, float beta2, float eps, float l2_reg,
                                float loss_scale, float* params_full_precision, uint16_t* params, float* gradients, float* first_moments,
                                float* second_moments, uint32_t* param_steps, int clear_grid_gradients, const float* lr_table,
                                uint32_t table_len, void* stream);

/* Adam on fp16 gradients (the reference's format and loss-scaled values), as adam_step_kernel;
 * lr_table optional (table_len 0).  Replaces step_optimizer (ngp.train.cu:1973-1980) for callers
 * that keep fp16 gradients. */
NGP_API int ngp_adam_step_f16(uint32_t n_params, uint32_t n_mlp, float lr, float beta1, float beta2, float eps, float l2_reg, float loss_scale,
                              float* params_full_precision, uint16_t* params, const uint16_t* gradients, float* first_moments,
                              float* second_moments, uint32_t* param_steps, const float* lr_table, uint32_t table_len, void* stream);

/* ngp_adam_step_f16 on the range [first, first + count) of the packed vector (one rank's shard
 * of the data-parallel exchange): every pointer points at element `first`; first is a multiple
 * of 4; elements with packed index < n_mlp are the dense MLP weights.  Replaces the part of
 * adam_step_kernel (ngp.train.cu:1261-1280) that this rank owns. */
NGP_API int ngp_adam_step_f16_range(uint32_t count, uint32_t first, uint32_t n_mlp, float lr, float beta1, float beta2, float eps, float l2_reg,
                                    float loss_scale, float* params_full_precision, uint16_t* params, const uint16_t* gradients,
                                    float* first_moments, float* second_moments, uint32_t* param_steps, const float* lr_table,
                                    uint32_t table_len, void* stream);

/* fp32 gradients -> fp16 (round to nearest); clear != 0 zeroes the fp32 source.  Both buffers
 * 16-byte aligned.  (The conversion before the data-parallel exchange, ngp.train.cpp:123-124.) */
NGP_API int ngp_gradients_to_half(uint32_t n, float* gradients, uint16_t* out, int clear, void* stream);

/* ------------------------------------------------------------------------------------------
 * Parameter initialisation (the reference's seeds and order).
 * ------------------------------------------------------------------------------------------ */
/* Replaces initialize_mlp_parameters (ngp.train.cu:1423-1461): the 10,240 MLP weights,
 * Xavier-uniform per matrix from PCG32 seed 1337, fp32 master + fp16 copy (synchronous). */
NGP_API int ngp_init_mlp_parameters(float* master, uint16_t* params, void* stream);
/* Replaces initialize_grid_params_kernel (ngp.train.cu:1002-1017): n_grid values U(-1e-4, 1e-4). */
NGP_API int ngp_init_grid_parameters(uint32_t n_grid, float* master_grid, uint16_t* params_grid, void* stream);
/* fp32 -> fp16 copy (cast_params_to_half_kernel). */
NGP_API int ngp_cast_to_half(uint32_t n, const float* in, uint16_t* out, void* stream);

/* ------------------------------------------------------------------------------------------
 * Trainer: the reference's ngp::train::InstantNGP (ngp.train.ixx:40-53) as an opaque handle.
 * ------------------------------------------------------------------------------------------ */
typedef struct ngp_trainer ngp_trainer;

typedef struct ngp_trainer_config {
    uint32_t n_levels, features_per_level, log2_hashmap_size, base_resolution;
    double log2_per_level_scale;
    float learning_rate;
} ngp_trainer_config;

/* One dataset split on the host: RGBA8 pixels [frames][height][width][4], cameras [frames][12]. */
typedef struct ngp_split {
    const uint8_t* pixels;
    const float* camera;
    uint32_t frame_count, width, height;
    float focal_x, focal_y, principal_x, principal_y;
} ngp_split;

/* TrainStats (ngp.train.ixx:8-18). */
typedef struct ngp_train_stats {
    uint32_t step, rays_per_batch, measured_sample_count_before_compaction, measured_sample_count, density_grid_occupied_cells;
    float loss, elapsed_ms, density_grid_update_ms, density_grid_occupancy_ratio;
} ngp_train_stats;

NGP_API void ngp_trainer_default_config(ngp_trainer_config* cfg);
/* Upload the splits, allocate and initialise everything (InstantNGP::InstantNGP, ngp.train.cpp:12-100). */
NGP_API int ngp_trainer_create(const ngp_trainer_config* cfg, const ngp_split* train, const ngp_split* validation, const ngp_split* test,
                               ngp_trainer** out);
NGP_API void ngp_trainer_destroy(ngp_trainer* t);
/* InstantNGP::train(iters) (ngp.train.cpp:108-155). */
NGP_API int ngp_trainer_train(ngp_trainer* t, int32_t iters, ngp_train_stats* stats);
/* Render `image_count` images of split 1 (validation) or 2 (test) and sum the squared error;
 * comparison_host (optional, one image only) receives [height][2*width][3] RGB8.
 * InstantNGP::validate / test (ngp.train.cpp:157-229). */
NGP_API int ngp_trainer_evaluate(ngp_trainer* t, int split, uint32_t image_begin, uint32_t image_count, uint8_t* comparison_host,
                                 double* out_sse, uint64_t* out_pixels);
/* Render a novel view (camera: 12 floats, host) into rgb_device [height*width][3] (fp32, [0,1]). */
NGP_API int ngp_trainer_render(ngp_trainer* t, const float* camera_host, uint32_t width, uint32_t height, float fx, float fy, float cx,
                               float cy, float* rgb_device);
/* ngp_trainer_render of a set of 64 x 64 image tiles: tiles first_tile, first_tile + tile_stride,
 * ... of the row-major tile grid (ceil(width / 64) tiles per row; the right and bottom tiles are
 * clipped to the image).  Only those tiles' pixels of rgb_device are written.  The tile loop of the
 * reference's run_evaluation (ngp.train.cu:1616-1620) partitioned across GPUs: rank r of N renders
 * tiles r, r + N, ... with no collective. */
NGP_API int ngp_trainer_render_tiles(ngp_trainer* t, const float* camera_host, uint32_t width, uint32_t height, float fx, float fy, float cx, float cy,
                                     uint32_t first_tile, uint32_t tile_stride, float* rgb_device);
/* Evaluation and rendering by segmented marching (enabled != 0, the default: rays are marched a
 * segment at a time and no further than their transmittance lasts) or, as the reference does,
 * by marching every occupied step of each tile before the network runs (0).  Both give the same
 * images bit for bit.  run_evaluation (ngp.train.cu:1597-1658). */
NGP_API int ngp_trainer_set_segmented_eval(ngp_trainer* t, int enabled);
/* The adaptive batch of the next step from this step's counts (InstantNGP::train,
 * ngp.train.cpp:132-133): inference samples = pre-compaction count (at most MAX_SAMPLES) rounded
 * up to 128; rays = rays * 2^18 / compacted count (at most 2^18), rounded up to 128, within
 * [128, 2^18].  Host-only arithmetic. */
NGP_API void ngp_adaptive_batch(uint32_t rays_per_batch, uint32_t measured_before, uint32_t measured, uint32_t* next_rays,
                                uint32_t* next_inference_samples);
NGP_API uint32_t ngp_trainer_param_count(const ngp_trainer* t);
/* fp32 master parameters [MLP | grid] to / from the host (export_weights / load_weights;
 * loading resets the optimizer and is allowed only before training, ngp.train.cpp:312). */
NGP_API int ngp_trainer_get_params(ngp_trainer* t, float* host_out, uint32_t count);
NGP_API int ngp_trainer_set_params(ngp_trainer* t, const float* host_in, uint32_t count);
/* Data parallelism over NVLink (no counterpart in the single-GPU reference; hooks between
 * backward_network and step_optimizer, ngp.train.cpp:123-124).  Rank 0 creates an NCCL unique id
 * (ngp_nccl_unique_id, 128 bytes), the caller shares it with every rank, and each rank's trainer
 * joins before its first step.  Each rank then marches its own rays (PCG32 stream step*world +
 * rank); per step the fp32 gradients are rounded to fp16 (loss-scaled, the reference's gradient
 * format) and reduce-scattered, each rank takes the Adam step on its 1/world shard, and the fp16
 * parameters are all-gathered (replicas stay bit-identical).  The communicator is non-blocking:
 * a collective, or a wait for the stream that runs it, that does not complete within the
 * collective timeout (default 120 s, $NGP_COLLECTIVE_TIMEOUT_MS, or
 * ngp_trainer_set_collective_timeout) aborts the communicator and returns NGP_ERR_TIMEOUT; an
 * asynchronous NCCL error aborts it and returns NGP_ERR_CUDA.  After a data-parallel join,
 * ngp_trainer_get_params is a collective (every rank calls it). */
NGP_API int ngp_nccl_unique_id(uint8_t* out, size_t bytes);
NGP_API int ngp_trainer_join(ngp_trainer* t, const uint8_t* unique_id, int world, int rank);
NGP_API int ngp_trainer_set_collective_timeout(ngp_trainer* t, double timeout_ms);
/* The gradient exchange a joined trainer uses: 0 none (not joined), 1 NCCL reduce-scatter +
 * Adam on the shard + all-gather, 2 the same three steps in one kernel over NVLink peer memory
 * (the default when every rank can map every peer's buffers; $NGP_EXCHANGE=nccl selects 1). */
NGP_API int ngp_trainer_exchange_mode(const ngp_trainer* t);
/* Training loss (no reference counterpart; the reference trains with L2, ngp.train.cu:817-820):
 * 0 = L2 (default), 1 = Huber (as ngp_training_loss_selected_kind). */
NGP_API int ngp_trainer_set_loss(ngp_trainer* t, int loss_kind);
/* Per-phase device time of the training step, summed over the steps since profiling was
 * enabled (cudaEvents between phases): 0 grid update, 1 ray marching, 2 density evaluation of the
 * marched samples + compaction, 3 network forward of the compacted samples + loss + padding,
 * 4 network backward, 5 encoding backward, 6 gradient exchange (fp16 conversion +
 * reduce-scatter), 7 Adam (+ all-gather of the fp16 parameters).  out_ms needs 8 floats;
 * out_mean_inference_samples = mean marched samples per step. */
/* Run-ahead (on by default; no counterpart in the reference): when the step after a train call
 * updates the density grid, the call leaves that update's first half (samples, encoding, density
 * network and splat into internal scratch) running on the GPU when it returns, so the GPU is not
 * idle while the host enters the next call; the next step completes the update.  Nothing a caller
 * can observe changes before that step.  A call's elapsed_ms then covers its steps without the
 * first half of its first step's update when the previous call ran it ahead: turn it off (which
 * also drops work already run ahead) to time exactly the work of a call's steps. */
NGP_API int ngp_trainer_set_run_ahead(ngp_trainer* t, int enable);

NGP_API int ngp_trainer_set_profiling(ngp_trainer* t, int enable);
NGP_API int ngp_trainer_phase_times(const ngp_trainer* t, float* out_ms, uint32_t n, uint32_t* out_steps, float* out_mean_inference_samples);
/* Profiled grid updates (no reference counterpart; update_density_grid, ngp.train.cu:1526-1595,
 * split by kernel): accumulated ms of [0] sample generation, [1] encoding, [2] density network,
 * [3] splat, [4] EMA + mean + bitfield (n >= 5), the number of updates and their mean sample count. */
NGP_API int ngp_trainer_grid_phase_times(const ngp_trainer* t, float* out_ms, uint32_t n, uint32_t* out_updates, float* out_mean_samples);
/* Occupancy bitfield (2^18 bytes) and density-grid values (2^21 floats) to the host. */
NGP_API int ngp_trainer_get_grid(const ngp_trainer* t, uint8_t* bitfield_host, float* values_host);

#ifdef __cplusplus
}
#endif

#endif /* NGP_B200_H */
