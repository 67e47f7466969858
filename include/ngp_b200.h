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
 * symbol it stands in for.  The C++ header `ngp.train.h` in this directory re-exports the
 * reference's exact `ngp::cuda` signatures on top of these functions.
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

#define NGP_MAX_LEVELS 32
#define NGP_SAMPLE_FLOATS 7
#define NGP_RAY_FLOATS 6

/* Most recent error message of the calling host thread ("" if none). */
NGP_API const char* ngp_last_error(void);
/* Library version string. */
NGP_API const char* ngp_version(void);

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

/* Sticky device status of the MLP kernels: bit 0 = a tensor-core completion wait timed out.
 * reset != 0 clears it. */
NGP_API int ngp_mlp_status(uint32_t* out_status, int reset);

#ifdef __cplusplus
}
#endif

#endif /* NGP_B200_H */
