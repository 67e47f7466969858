// Trainer: owns every device buffer and runs the NeRF training step, validation and test
// rendering on one stream.  Mirrors the reference's ngp::train::InstantNGP
// (ngp.train.ixx:40-150, ngp.train.cpp:12-229): same step order, same adaptive batch rule,
// same statistics; the device work is the library's own kernels.
//
// Differences from the reference, all B200-motivated:
// * every buffer is sized once for the largest batch (no per-call attribute setting, no 2^18
//   chunking of the inference pass: one launch covers up to 2^22 samples);
// * the network forward of the compacted batch is not run: the backward recomputes its
//   activations on chip from the encoded inputs;
// * gradients are fp32 and Adam clears the grid gradient in the same pass;
// * evaluation marches 2^16-pixel tiles a segment at a time and stops marching a ray once its
//   transmittance is spent, instead of marching every occupied step of 4096-pixel tiles.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "sampler.cuh"

#include <nccl.h>

using namespace ngp;

namespace {

constexpr uint32_t kNoStep     = 0xFFFFFFFFu;
constexpr uint32_t kMlpParams  = 10240;
constexpr int kTrainPhases     = 8;  // see ngp_trainer_phase_times
constexpr int kGridPhases      = 5;  // see ngp_trainer_grid_phase_times
constexpr uint32_t kLrTableCapacity = 1u << 20;
constexpr uint32_t kLrTableBlock    = 4096u;
// Segmented evaluation: tiles of 2^16 pixel rays; the first segment marches at most
// MAX_SAMPLES / tile = 64 samples per ray (so it always fits), later ones 128, then the rest.
#ifndef NGP_SEG_TILE_LOG2
#define NGP_SEG_TILE_LOG2 16
#endif
#ifndef NGP_SEG_CAP1
#define NGP_SEG_CAP1 128
#endif
constexpr uint32_t kSegTile         = 1u << NGP_SEG_TILE_LOG2;
constexpr uint32_t kSegCaps[]       = {kMaxSamples / kSegTile, NGP_SEG_CAP1, kMarchSteps};

template <typename T>
int dalloc(T*& p, size_t count, const char* what) {
    p = nullptr;
    if (count == 0) return NGP_OK;
    if (fault_due(kFaultAlloc)) return fail(NGP_ERR_CUDA, std::string("cudaMalloc ") + what + ": injected fault (alloc)");
    void* raw           = nullptr;
    const cudaError_t e = cudaMalloc(&raw, count * sizeof(T));
    if (e != cudaSuccess) return fail(NGP_ERR_CUDA, std::string("cudaMalloc ") + what + ": " + cudaGetErrorString(e));
    p = static_cast<T*>(raw);
    return NGP_OK;
}

struct Split {
    uint8_t* pixels = nullptr;
    float* camera   = nullptr;
    uint32_t frames = 0, width = 0, height = 0;
    float fx = 0, fy = 0, cx = 0, cy = 0;
};

}  // namespace

#ifndef NGP_OVERLAP_MARCH
#define NGP_OVERLAP_MARCH 1  // 0: every step marches on its own stream (no cross-step overlap; measured 0.87 vs 0.75 ms)
#endif
#ifndef NGP_DP_PRIORITY
#define NGP_DP_PRIORITY 1  // 0: equal stream priorities; the all-reduce waits for the next step's march (measured 0.935 vs 0.914 ms at 4 GPUs)
#endif
#ifndef NGP_SELECT
#define NGP_SELECT 1  // 0: the kept samples' records and encodings are copied into a compacted batch
#endif

struct MarchSet {
    float* coords         = nullptr;  // [MAX_SAMPLES][7]
    float* rays           = nullptr;  // [BATCH][6]
    uint32_t* ray_indices = nullptr;
    uint32_t* numsteps    = nullptr;
    uint32_t* counters    = nullptr;  // 0 rays, 1 samples, 2 compacted
};

struct ngp_trainer {
    ngp_trainer_config cfg{};
    ngp_grid_layout layout{};
    cudaStream_t stream = nullptr;
    Split train, val, test;

    // parameters and optimizer
    uint32_t n_params = 0;
    float* master      = nullptr;
    uint16_t* params   = nullptr;
    float* grads       = nullptr;
    uint16_t* grads16  = nullptr;  // data parallel: fp16 gradient exchanged between ranks
    float *adam_m = nullptr, *adam_v = nullptr;
    uint32_t* adam_steps = nullptr;

    // density grid
    float *grid_values = nullptr, *grid_scratch = nullptr, *grid_partial = nullptr, *grid_mean = nullptr;
    uint32_t* grid_indices = nullptr;
    uint8_t* bitfield      = nullptr;
    uint32_t* occupied     = nullptr;
    uint32_t* grid_counter = nullptr;  // slot counter of the cell-ordered grid samples

    // sampler and network buffers
    // Two sets of march outputs, used by alternate steps, so that the next step's march can run
    // while this step's loss pass still reads its rays and sample counts; a third set serves
    // evaluation, so that a march launched for the next training step survives evaluation and
    // rendering calls between train calls.
    MarchSet sets[3];
    float* coords = nullptr;  // evaluation set: [MAX_SAMPLES][7]
    float* rays   = nullptr;  // evaluation set: [BATCH][6]
    uint32_t *ray_indices = nullptr, *numsteps = nullptr, *march_scratch = nullptr, *eval_march_scratch = nullptr;
    uint32_t* counters     = nullptr;  // evaluation set: 0 rays, 1 samples, 2 compacted
    uint16_t* enc          = nullptr;  // [32][MAX_SAMPLES] encoded positions
    uint16_t* out          = nullptr;  // [MAX_SAMPLES][16] network output (training: raw densities)
    uint32_t* rows         = nullptr;  // [MAX_SAMPLES] row list of the progressive density evaluation
    uint32_t* batch_rows   = nullptr;  // [COMPACTED_ROWS] the batch as rows of the kept samples
    uint16_t* dens         = nullptr;  // [MAX_SAMPLES] raw densities of the evaluated samples
    uint16_t* cout         = nullptr;  // [COMPACTED_ROWS][16] network output of the compacted samples
    uint16_t* grid_density = nullptr;  // [2^21] raw density of the grid samples
    float* ccoords         = nullptr;  // [COMPACTED_ROWS][7] compacted
    uint16_t* dloss        = nullptr;  // [BATCH][16]
    float* loss_values     = nullptr;  // [BATCH]
    unsigned char* loss_scratch = nullptr;
    size_t loss_scratch_bytes   = 0;
    uint16_t* cenc   = nullptr;  // [32][COMPACTED_ROWS] encoded compacted samples
    uint16_t* denc   = nullptr;  // [32][BATCH] dL/d(encoding)
    float* mlp_scratch        = nullptr;
    size_t mlp_scratch_floats = 0;
    double* eval_sse          = nullptr;
    uint8_t* comparison       = nullptr;
    // segmented evaluation (tiles of kSegTile pixels): per-ray state carried between segments
    bool eval_segmented    = true;
    float* seg_tout        = nullptr;  // [tile entry] where the ray continues
    float* seg_tstate      = nullptr;  // [tile ray]
    uint32_t* seg_marched  = nullptr;  // [tile ray]
    float* seg_state       = nullptr;  // [tile ray][4] T, r, g, b
    uint32_t* seg_lists    = nullptr;  // [2][tile] ray lists of alternate segments
    uint32_t* seg_counters = nullptr;  // 0 samples, 1 fitted entries, 2/3 list counts of alternate segments
    uint32_t* seg_host     = nullptr;  // pinned copy of seg_counters

    // host state (ngp.train.ixx:79-89)
    uint32_t step              = 0;
    // data parallelism: one trainer per GPU, rays split by rank, gradients all-reduced
    ncclComm_t comm = nullptr;
    int world = 1, rank = 0;
    // the gradient exchange: fp16 gradients [n_padded] are reduce-scattered, each rank's Adam
    // updates its shard [rank * shard, rank * shard + shard) and the fp16 parameters [n_padded]
    // are all-gathered; n_padded = n_params rounded up to a multiple of 4 * world
    uint32_t n_padded = 0, shard = 0;
    // a collective (or a wait on a stream that runs one) that takes longer fails: the
    // communicator is aborted and the call returns NGP_ERR_TIMEOUT
    double collective_timeout_ms = 120000.0;
    // fused exchange over NVLink peer memory (peer_exchange_adam): the ranks' fp16 gradient,
    // fp16 parameter and flag buffers mapped into this process (CUDA IPC); used when every rank
    // could map every peer, else the NCCL reduce-scatter / all-gather path
    bool peer_exchange       = false;
    uint32_t* peer_flags     = nullptr;  // this rank's 2 * world flags + CTA counter
    void** peer_table        = nullptr;  // device: [3][world] grads, params, flags
    std::vector<void*> peer_opened;      // IPC mappings to close
    uint32_t peer_epoch      = 0;
    uint32_t* peer_status    = nullptr;  // device error word of the fused exchange
    int loss_kind                = 0;  // 0 L2 (the reference's), 1 Huber
    // optional per-phase timing (cudaEvents between the phases of a step)
    bool profiling = false;
    cudaEvent_t marks[kTrainPhases + 1] = {};
    double phase_ms[kTrainPhases]       = {};
    double inference_samples_sum        = 0.0;
    uint32_t profiled_steps             = 0;
    uint32_t rays_per_batch    = 1u << 12;
    uint32_t inference_samples = kMaxSamples;
    uint32_t measured_before = 0, measured = 0;
    uint32_t ema_step       = 0;
    uint32_t occupied_cells = 0;
    float grid_update_ms    = 0.0f;
    // Cross-step pipelining inside one train call: once a step's loss pass has produced its
    // counters, the next step's rays are marched on march_stream while this step's backward and
    // optimizer run (marching reads only the bitfield, which changes only on grid-update steps).
    cudaStream_t march_stream = nullptr;
    cudaEvent_t ev_counts = nullptr, ev_march = nullptr;
    uint32_t* host_counters = nullptr;  // pinned copy of counters 0..4
    bool one_round          = false;    // progressive evaluation in one round (see train_step)
    uint32_t grid_begun     = 0xFFFFFFFFu;  // step whose grid update's first half is already enqueued
    uint32_t grid_samples_pending = 0;      // samples of the update begun last
    bool run_ahead          = true;         // see begin_next_grid_update
    float* host_loss        = nullptr;  // pinned copy of the last step's per-ray loss [BATCH]
    bool premarched         = false;    // step `step` was marched on march_stream
    // Adam: bias-corrected rate per step count, entries [1, lr_table_len] filled
    float* lr_table       = nullptr;
    uint32_t lr_table_len = 0;
    uint32_t adam_calls   = 0;  // bounds every parameter's step count
    // grid-update timing: a pool of event pairs created once and reused by every train call
    // (grid_events_used pairs are pending in the current call)
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> grid_events;
    size_t grid_events_used = 0;
    // profiling: events around the kernels of a grid update (samples, encode, density network,
    // splat, EMA + mean + bitfield), their accumulated times and the samples they processed
    cudaEvent_t grid_marks[kGridPhases + 1] = {};
    double grid_phase_ms[kGridPhases]       = {};
    double grid_samples_sum                 = 0.0;
    uint32_t profiled_grid_updates          = 0;
};

namespace {

void free_split(Split& s) {
    cudaFree(s.pixels);
    cudaFree(s.camera);
    s = Split{};
}

void destroy(ngp_trainer* t) {
    if (t == nullptr) return;
    if (t->stream) cudaStreamSynchronize(t->stream);
    free_split(t->train);
    free_split(t->val);
    free_split(t->test);
    void* ptrs[] = {t->master, t->params, t->grads, t->grads16, t->adam_m, t->adam_v, t->adam_steps, t->grid_values, t->grid_scratch, t->grid_partial,
                    t->grid_mean, t->grid_indices, t->bitfield, t->occupied, t->grid_counter, t->march_scratch, t->eval_march_scratch, t->enc, t->out, t->rows, t->batch_rows, t->dens, t->cout, t->grid_density, t->ccoords, t->dloss, t->loss_values, t->loss_scratch, t->cenc, t->denc,
                    t->mlp_scratch, t->eval_sse, t->comparison, t->lr_table, t->seg_tout, t->seg_tstate, t->seg_marched, t->seg_state,
                    t->seg_lists, t->seg_counters};
    for (void* p : ptrs) cudaFree(p);
    for (MarchSet& m : t->sets) cudaFree(m.coords), cudaFree(m.rays), cudaFree(m.ray_indices), cudaFree(m.numsteps), cudaFree(m.counters);
    for (void* q : t->peer_opened) cudaIpcCloseMemHandle(q);
    cudaFree(t->peer_flags), cudaFree(t->peer_table), cudaFree(t->peer_status);
    if (t->comm) {
        // non-blocking communicator: finalize (bounded wait), then destroy; abort if it hangs
        const ncclResult_t fr = ncclCommFinalize(t->comm);
        bool finalized        = fr == ncclSuccess || fr == ncclInProgress;
        const auto start      = std::chrono::steady_clock::now();
        ncclResult_t a        = ncclInProgress;
        while (finalized && a == ncclInProgress) {
            ncclCommGetAsyncError(t->comm, &a);
            if (std::chrono::steady_clock::now() - start > std::chrono::seconds(10)) finalized = false;
        }
        if (finalized && a == ncclSuccess)
            ncclCommDestroy(t->comm);
        else
            ncclCommAbort(t->comm);
    }
    if (t->march_stream) cudaStreamSynchronize(t->march_stream);
    for (cudaEvent_t e : t->marks)
        if (e) cudaEventDestroy(e);
    for (auto& pr : t->grid_events) cudaEventDestroy(pr.first), cudaEventDestroy(pr.second);
    for (cudaEvent_t e : t->grid_marks)
        if (e) cudaEventDestroy(e);
    if (t->ev_counts) cudaEventDestroy(t->ev_counts);
    if (t->ev_march) cudaEventDestroy(t->ev_march);
    if (t->host_counters) cudaFreeHost(t->host_counters);
    if (t->host_loss) cudaFreeHost(t->host_loss);
    if (t->seg_host) cudaFreeHost(t->seg_host);
    if (t->march_stream) cudaStreamDestroy(t->march_stream);
    if (t->stream) cudaStreamDestroy(t->stream);
    delete t;
}

int upload_split(Split& s, const ngp_split* in, const char* what) {
    s = Split{};
    if (in == nullptr || in->frame_count == 0) return NGP_OK;
    if (in->pixels == nullptr || in->camera == nullptr || in->width == 0 || in->height == 0 || !(in->focal_x > 0) || !(in->focal_y > 0))
        return fail(NGP_ERR_INVALID, std::string("invalid dataset split: ") + what);
    const size_t pix = static_cast<size_t>(in->frame_count) * in->width * in->height * 4u;
    NGP_TRY(dalloc(s.pixels, pix, "dataset pixels"));
    NGP_TRY(dalloc(s.camera, static_cast<size_t>(in->frame_count) * 12u, "dataset cameras"));
    NGP_TRY(check_cuda(cudaMemcpy(s.pixels, in->pixels, pix, cudaMemcpyHostToDevice), "upload pixels"));
    NGP_TRY(check_cuda(cudaMemcpy(s.camera, in->camera, sizeof(float) * in->frame_count * 12u, cudaMemcpyHostToDevice), "upload cameras"));
    s.frames = in->frame_count, s.width = in->width, s.height = in->height;
    s.fx = in->focal_x, s.fy = in->focal_y, s.cx = in->principal_x, s.cy = in->principal_y;
    return NGP_OK;
}

// U(-1e-4, 1e-4) grid entries from PCG32(1337) advanced past the MLP weights, four values per
// thread slot, as the reference's initialize_grid_params_kernel draws them (ngp.train.cu:1002-1017).
__global__ void init_grid_kernel(float* master, __half* params, uint32_t n_grid, uint32_t mlp_count) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x, n_threads = blockDim.x * gridDim.x;
    Pcg32 rng{kTrainSeed};
    rng.advance(static_cast<uint64_t>(mlp_count) + static_cast<uint64_t>(i) * 4u);
    for (uint32_t j = 0; j < 4; ++j) {
        const uint32_t idx = i + n_threads * j;
        if (idx >= n_grid) return;
        const float v = __fmaf_rn(rng.next_float(), 2e-4f, -1e-4f);
        master[idx]   = v;
        params[idx]   = __float2half_rn(v);
    }
}

__global__ void cast_half_kernel(const float* in, __half* out, uint32_t n) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __float2half_rn(in[i]);
}

// Xavier-uniform MLP weights drawn on the host from PCG32(1337), in the reference's order
// (ngp.train.cu:1423-1461).
int init_params(ngp_trainer* t) {
    NGP_TRY(ngp_init_mlp_parameters(t->master, t->params, t->stream));
    return ngp_init_grid_parameters(t->layout.n_params, t->master + kMlpParams, t->params + kMlpParams, t->stream);
}

int encode(ngp_trainer* t, uint32_t n, const float* c, uint16_t* dst, uint32_t stride) {
    return ngp_encode_grid_forward(&t->layout, n, c, 7, t->params + kMlpParams, dst, stride, t->stream);
}

// Grid-update schedule of update_density_grid (ngp.train.cu:1526-1531).
bool grid_update_due(uint32_t step) {
    uint32_t skip = step / 16u;
    skip          = skip < 1u ? 1u : (skip > 16u ? 16u : skip);
    return step % skip == 0u;
}

void grid_mark(ngp_trainer* t, int k) {
    if (t->profiling) cudaEventRecord(t->grid_marks[k], t->stream);
}

// First half of a grid update: the samples, their encodings and the density network with the
// splat into the grid scratch.  It writes only internal buffers (encodings, cell indices, grid
// samples and the scratch the previous update's bitfield pass cleared), so it can run ahead of
// the step that completes the update (begin_next_grid_update).
int grid_update_begin(ngp_trainer* t) {
    const Split& s = t->train;
    if (t->step == 0) {
        t->ema_step = 0;
        NGP_TRY(ngp_density_grid_mark_untrained(s.camera, s.frames, s.width, s.height, s.fx, s.fy, s.cx, s.cy, t->grid_values, t->stream));
    }
    const uint32_t n_uniform = t->step < 256u ? kGridCells : kGridCells / 4u;
    const uint32_t n_nonuni  = t->step < 256u ? 0u : kGridCells / 4u;
    const uint32_t n         = n_uniform + n_nonuni;
    float* coords = t->sets[t->step & 1u].coords;
    // the reference's samples in Morton cell order (the encoding below then gathers neighbouring
    // table entries); the splat's atomic max does not depend on their order.  In the warm-up (all
    // 2^21 samples uniform) the samples are made inside the encoding kernel.
    if (n_nonuni == 0 && n_uniform == kGridCells) {
        grid_mark(t, 1);
        NGP_TRY(ngp_density_grid_encode_samples(&t->layout, t->ema_step, t->grid_values, t->params + kMlpParams, t->enc, n, t->grid_indices,
                                                t->stream));
    } else {
        NGP_TRY(ngp_density_grid_samples_cell_order(n_uniform, n_nonuni, t->ema_step, t->grid_values, coords, t->grid_indices, t->grid_counter,
                                                    t->stream));
        grid_mark(t, 1);
        NGP_TRY(encode(t, n, coords, t->enc, n));
    }
    grid_mark(t, 2);
    // density network with the splat (K3) in its epilogue: scratch[cell] = max(..., exp(d) * dt)
    NGP_TRY(ngp_density_forward_splat(n, t->params, t->enc, n, t->grid_indices, t->grid_scratch, t->stream));
    grid_mark(t, 3);
    t->grid_samples_pending = n;
    return NGP_OK;
}

// update_density_grid (ngp.train.cu:1526-1595).
int update_grid(ngp_trainer* t) {
    if (!grid_update_due(t->step)) return NGP_OK;
    const bool begun = t->grid_begun == t->step;  // the first half ran at the end of the last train call
    t->grid_begun    = kNoStep;
    cudaEvent_t ev_end = nullptr;
    if (!begun) {
        if (t->grid_events_used == t->grid_events.size()) {
            cudaEvent_t e0 = nullptr, e1 = nullptr;
            NGP_TRY(check_cuda(cudaEventCreate(&e0), "grid timing event"));
            if (const int st = check_cuda(cudaEventCreate(&e1), "grid timing event"); st != NGP_OK) {
                cudaEventDestroy(e0);
                return st;
            }
            t->grid_events.emplace_back(e0, e1);
        }
        const auto& ev = t->grid_events[t->grid_events_used++];
        cudaEventRecord(ev.first, t->stream);
        ev_end = ev.second;
        grid_mark(t, 0);
        NGP_TRY(grid_update_begin(t));
    }
    grid_mark(t, 4);
    NGP_TRY(ngp_density_grid_update(t->grid_values, t->grid_scratch, 0.95f, t->grid_partial, t->grid_mean, t->bitfield, t->occupied, t->stream));
    grid_mark(t, 5);
    ++t->ema_step;
    if (ev_end != nullptr) cudaEventRecord(ev_end, t->stream);
    if (t->profiling) {
        NGP_TRY(check_cuda(cudaEventSynchronize(t->grid_marks[kGridPhases]), "grid update"));
        for (int k = 0; k < kGridPhases; ++k) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, t->grid_marks[k], t->grid_marks[k + 1]);
            t->grid_phase_ms[k] += ms;
        }
        t->grid_samples_sum += t->grid_samples_pending;
        ++t->profiled_grid_updates;
    }
    return NGP_OK;
}

// At the end of a train call: when the next step updates the density grid, its first half goes
// onto the stream now, behind the call's last optimizer step, so that the GPU has that work while
// the host returns from this call and enters the next one.  Its results are consumed by the next
// step; set_params discards them.  (Not while profiling: the phase marks time whole updates.)
int begin_next_grid_update(ngp_trainer* t) {
    if (!t->run_ahead || t->profiling || t->step == 0 || !grid_update_due(t->step) || t->grid_begun == t->step) return NGP_OK;
    NGP_TRY(grid_update_begin(t));
    t->grid_begun = t->step;
    return NGP_OK;
}

// Drops a grid-update first half enqueued ahead (the parameters changed, or its phase marks are
// wanted): the scratch it splatted into is cleared again, and the step redoes it.
int discard_grid_begin(ngp_trainer* t) {
    if (t->grid_begun == kNoStep) return NGP_OK;
    t->grid_begun = kNoStep;
    return check_cuda(cudaMemsetAsync(t->grid_scratch, 0, sizeof(float) * kGridCells, t->stream), "discard grid update");
}

// Adds the finished grid updates' durations to grid_update_ms.
void collect_grid_times(ngp_trainer* t) {
    for (size_t i = 0; i < t->grid_events_used; ++i) {
        const auto& pr = t->grid_events[i];
        float ms       = 0.0f;
        if (cudaEventSynchronize(pr.second) == cudaSuccess && cudaEventElapsedTime(&ms, pr.first, pr.second) == cudaSuccess) t->grid_update_ms += ms;
    }
    t->grid_events_used = 0;
}

int march_step(ngp_trainer* t, uint32_t step, cudaStream_t stream) {
    const Split& s          = t->train;
    const uint32_t rng_step = step * static_cast<uint32_t>(t->world) + static_cast<uint32_t>(t->rank);
    const MarchSet& m       = t->sets[step & 1u];
    return ngp_march_training_rays(s.camera, s.frames, s.width, s.height, s.fx, s.fy, s.cx, s.cy, rng_step, t->rays_per_batch, nullptr,
                                   t->inference_samples, t->bitfield, m.coords, m.rays, m.ray_indices, m.numsteps, t->march_scratch,
                                   m.counters + 0, m.counters + 1, stream);
}

void mark(ngp_trainer* t, int k) {
    if (t->profiling) cudaEventRecord(t->marks[k], t->stream);
}

// ---- collectives with a host deadline ------------------------------------------------------
// The communicator is non-blocking (ncclCommInitRankConfig, blocking = 0): an NCCL call may
// return ncclInProgress while it is enqueued, and a peer that has left or hangs shows up as an
// asynchronous error or as a wait that never ends.  Every wait on a communicator (its
// initialisation, a call in progress, the stream that runs its kernels) polls
// ncclCommGetAsyncError until the trainer's collective timeout; on expiry or error the
// communicator is aborted (ncclCommAbort ends its kernels) and the call returns an error.
int abort_comm(ngp_trainer* t, int code, const std::string& message) {
    if (t->comm != nullptr) {
        ncclCommAbort(t->comm);
        t->comm = nullptr;
    }
    return fail(code, message);
}

template <typename Done>
int wait_comm(ngp_trainer* t, Done&& done, const char* what) {
    const auto start = std::chrono::steady_clock::now();
    for (uint32_t spin = 0;; ++spin) {
        const int d = done();
        if (d > 0) return NGP_OK;
        if (d < 0) return abort_comm(t, NGP_ERR_CUDA, std::string(what) + ": " + ngp_last_error());
        if (t->comm != nullptr) {
            ncclResult_t async = ncclSuccess;
            ncclCommGetAsyncError(t->comm, &async);
            if (async != ncclSuccess && async != ncclInProgress)
                return abort_comm(t, NGP_ERR_CUDA, std::string(what) + ": NCCL error " + ncclGetErrorString(async) + "; communicator aborted");
        }
        const double ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - start).count();
        if (ms > t->collective_timeout_ms)
            return abort_comm(t, NGP_ERR_TIMEOUT, std::string(what) + ": not complete after " + std::to_string(static_cast<long long>(ms)) +
                                                    " ms (a peer rank may have left); communicator aborted");
        if (spin > 64) std::this_thread::sleep_for(std::chrono::microseconds(spin > 4096 ? 200 : 5));
    }
}

// Waits for an event recorded on a stream that may run collectives (plain synchronisation when
// the trainer has no communicator).
int wait_event(ngp_trainer* t, cudaEvent_t ev, const char* what) {
    if (t->comm == nullptr) return check_cuda(cudaEventSynchronize(ev), what);
    return wait_comm(t, [&]() -> int {
        const cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return 1;
        if (e == cudaErrorNotReady) return 0;
        check_cuda(e, what);
        return -1;
    }, what);
}

int wait_stream(ngp_trainer* t, cudaStream_t s, const char* what) {
    if (t->comm == nullptr) return check_cuda(cudaStreamSynchronize(s), what);
    return wait_comm(t, [&]() -> int {
        const cudaError_t e = cudaStreamQuery(s);
        if (e == cudaSuccess) return 1;
        if (e == cudaErrorNotReady) return 0;
        check_cuda(e, what);
        return -1;
    }, what);
}

// Result of an NCCL call on the non-blocking communicator: waits while it is in progress.
int nccl_done(ngp_trainer* t, ncclResult_t r, const char* what) {
    if (fault_due(kFaultCollective)) return abort_comm(t, NGP_ERR_CUDA, std::string(what) + ": injected fault (collective)");
    if (r == ncclSuccess) return NGP_OK;
    if (r != ncclInProgress) return abort_comm(t, NGP_ERR_CUDA, std::string(what) + ": " + ncclGetErrorString(r) + "; communicator aborted");
    return wait_comm(t, [&]() -> int {
        ncclResult_t a = ncclSuccess;
        ncclCommGetAsyncError(t->comm, &a);
        if (a == ncclSuccess) return 1;
        if (a == ncclInProgress) return 0;
        set_error(ncclGetErrorString(a));
        return -1;
    }, what);
}

// One training step.  `premarch_next`: march step + 1 on march_stream once this step's counters
// are known (the caller guarantees that step + 1 follows in the same call).
int train_step(ngp_trainer* t, bool premarch_next) {
    const Split& s = t->train;
    mark(t, 0);
    if (t->premarched) {
        // marched during the previous step's backward pass (no grid update is due at this step)
        NGP_TRY(check_cuda(cudaStreamWaitEvent(t->stream, t->ev_march, 0), "wait march"));
        t->premarched = false;
        mark(t, 1);
    } else {
        NGP_TRY(update_grid(t));
        mark(t, 1);
        // sample_training_batch (ngp.train.cu:1919-1930)
        // each rank draws its rays from its own PCG32 stream; rank 0 of a single-GPU run uses the
        // reference's stream (step << 32)
        NGP_TRY(march_step(t, t->step, t->stream));
    }
    const uint32_t rng_step = t->step * static_cast<uint32_t>(t->world) + static_cast<uint32_t>(t->rank);
    mark(t, 2);
    // evaluate_network over the pre-compaction samples (ngp.train.cu:1494-1524) and compaction
    // (1932-1944): only the densities decide which samples a ray keeps, and only the samples in
    // front of each ray's stopping point need them
    const MarchSet& m = t->sets[t->step & 1u];
#if NGP_SELECT
    // the batch is a list of the kept samples' rows; the samples stay in place
    // one evaluation round when most rays outlived the first window in the previous step
    // (the first steps: low densities stop few rays); the selection is the same either way
    NGP_TRY(ngp_training_select_progressive_window(t->rays_per_batch, m.counters + 0, &t->layout, t->params, m.coords, t->inference_samples,
                                                   m.numsteps, t->enc, t->inference_samples, t->dens, t->rows, t->batch_rows, m.counters + 3,
                                                   m.counters + 2,
                                            t->loss_scratch, t->loss_scratch_bytes, t->one_round ? 0xFFFFFFFFu : 48u, m.counters + 4, t->stream));
#else
    NGP_TRY(ngp_training_compact_progressive(t->rays_per_batch, m.counters + 0, &t->layout, t->params, m.coords, t->inference_samples, m.numsteps,
                                             t->enc, t->inference_samples, t->dens, t->rows, t->ccoords, t->cenc, m.counters + 2, t->loss_scratch,
                                             t->loss_scratch_bytes, t->stream));
#endif
    // the step's counters are final here: the host reads them (for the next step's batch size)
    // while the rest of the step runs
    NGP_TRY(check_cuda(cudaMemcpyAsync(t->host_counters, m.counters, 5 * sizeof(uint32_t), cudaMemcpyDeviceToHost, t->stream), "read counters"));
    NGP_TRY(check_cuda(cudaEventRecord(t->ev_counts, t->stream), "record counters"));
    mark(t, 3);
    // the full network on the kept samples, then compositing, loss and padding (1944-1956)
#if NGP_SELECT
    NGP_TRY(ngp_mlp_forward_rows(kCompactedRows, t->batch_rows, m.counters + 3, t->params, t->enc, t->inference_samples, m.coords, 7, t->out,
                                 t->stream));
    NGP_TRY(ngp_training_loss_selected_kind(t->rays_per_batch, rng_step, m.counters + 0, s.pixels, s.frames, s.width, s.height, t->out,
                                            m.ray_indices, m.rays, m.numsteps, m.coords, t->dloss, t->loss_values, t->loss_scratch,
                                            t->loss_scratch_bytes, t->loss_kind, t->stream));
    NGP_TRY(ngp_pad_training_rows(m.counters + 2, t->batch_rows, t->dloss, t->stream));
    mark(t, 4);
    NGP_TRY(ngp_mlp_backward_rows(kNetworkBatch, t->batch_rows, t->params, t->enc, t->inference_samples, m.coords, 7, t->dloss, t->denc, kNetworkBatch,
                                  t->mlp_scratch, t->mlp_scratch_floats, t->grads, nullptr, 1.0f, t->stream));
    mark(t, 5);
    NGP_TRY(ngp_encode_grid_backward_rows(&t->layout, kNetworkBatch, t->batch_rows, m.coords, 7, t->denc, kNetworkBatch, t->grads + kMlpParams,
                                          t->stream));
    mark(t, 6);
#else
    NGP_TRY(ngp_mlp_forward(kCompactedRows, t->params, t->cenc, kCompactedRows, t->ccoords, 7, t->cout, nullptr, t->stream));
    NGP_TRY(ngp_training_loss_compacted(t->rays_per_batch, rng_step, m.counters + 0, s.pixels, s.frames, s.width, s.height, t->cout, m.ray_indices,
                                        m.rays, m.numsteps, t->ccoords, t->dloss, t->loss_values, t->loss_scratch, t->loss_scratch_bytes,
                                        t->stream));
    NGP_TRY(ngp_pad_training_batch_enc(m.counters + 2, t->ccoords, t->dloss, t->cenc, kCompactedRows, t->stream));
    mark(t, 4);
    NGP_TRY(ngp_mlp_backward(kNetworkBatch, t->params, t->cenc, kCompactedRows, t->ccoords, 7, t->dloss, t->denc, kNetworkBatch, t->mlp_scratch,
                             t->mlp_scratch_floats, t->grads, nullptr, 1.0f, t->stream));
    mark(t, 5);
    NGP_TRY(ngp_encode_grid_backward(&t->layout, kNetworkBatch, t->ccoords, 7, t->denc, kNetworkBatch, t->grads + kMlpParams, t->stream));
    mark(t, 6);
#endif
    // adaptive batch (ngp.train.cpp:125-133): this step's counters were copied after the loss
    // pass; the host waits for them while the backward pass runs, then launches the next step's
    // march on march_stream
    NGP_TRY(wait_event(t, t->ev_counts, "train step counters"));
    const uint32_t c[3] = {t->host_counters[0], t->host_counters[1], t->host_counters[2]};
    t->measured_before  = c[1];
    t->measured         = c[2];
    // rays still going after the first evaluation window (counter 4; 0 after a one-round step,
    // which keeps the next step on one round only while at least 70 % of the rays outlived it)
    if (!t->one_round) t->one_round = static_cast<uint64_t>(t->host_counters[4]) * 10u >= static_cast<uint64_t>(c[0]) * 7u && c[0] > 0;
    else if (t->step % 16u == 15u) t->one_round = false;  // look again every 16 steps
    if (t->measured == 0u) {
        cudaMemcpy(&t->occupied_cells, t->occupied, sizeof(uint32_t), cudaMemcpyDeviceToHost);
        return fail(NGP_ERR_STATE, "Training stopped unexpectedly. density_grid_occupied_cells=" + std::to_string(t->occupied_cells));
    }
    const uint32_t next_step   = t->step + 1u;
    uint32_t next_rays = 0, next_infer = 0;
    ngp_adaptive_batch(t->rays_per_batch, t->measured_before, t->measured, &next_rays, &next_infer);
    const bool premarch        = NGP_OVERLAP_MARCH && premarch_next && !t->profiling && !grid_update_due(next_step);
    if (premarch) {
        // the march writes the other set of march outputs, last read by the previous step (which
        // ev_counts follows in stream order)
        t->rays_per_batch    = next_rays;
        t->inference_samples = next_infer;
        NGP_TRY(check_cuda(cudaStreamWaitEvent(t->march_stream, t->ev_counts, 0), "march after loss"));
        NGP_TRY(march_step(t, next_step, t->march_stream));
        NGP_TRY(check_cuda(cudaEventRecord(t->ev_march, t->march_stream), "record march"));
    }
    // data parallel: the fp32 gradients are rounded to fp16 (the reference's gradient format,
    // loss-scaled by 128: half the bytes of fp32; the fp32 accumulation buffer is cleared by the
    // conversion) and reduce-scattered: each rank receives the sum over ranks of its shard, takes
    // the Adam step on that shard only, and the fp16 parameters are all-gathered, so every
    // replica (and the density grid it builds from them) stays identical.
    // NCCL's kernels must not wait for SM slots behind a long-running kernel of another stream (a
    // delayed rank stalls every rank): the training stream has the higher priority, so its
    // collectives are scheduled before the next step's march blocks.
    if (t->comm != nullptr) {
        if (premarch && !NGP_DP_PRIORITY) NGP_TRY(check_cuda(cudaStreamWaitEvent(t->stream, t->ev_march, 0), "exchange after march"));
        NGP_TRY(ngp_gradients_to_half(t->n_params, t->grads, t->grads16, 1, t->stream));
        if (!t->peer_exchange) {
            uint16_t* mine = t->grads16 + static_cast<size_t>(t->rank) * t->shard;
            NGP_TRY(nccl_done(t, ncclReduceScatter(t->grads16, mine, t->shard, ncclHalf, ncclSum, t->comm, t->stream), "ncclReduceScatter"));
        }
    }
    mark(t, 7);
    // step_optimizer (ngp.train.cu:1973-1980)
    if (t->adam_calls + 1u > t->lr_table_len) {
        // extend the bias-corrected rate table by a block of step counts
        const uint32_t first = t->lr_table_len + 1u, count = std::min(kLrTableBlock, kLrTableCapacity - first);
        if (count > 0) {
            NGP_TRY(ngp_adam_lr_table(t->lr_table, first, count, t->cfg.learning_rate, 0.9f, 0.99f, t->stream));
            t->lr_table_len += count;
        }
    }
    ++t->adam_calls;
    if (t->comm != nullptr && t->peer_exchange) {
        // reduce-scatter, Adam on this rank's shard and all-gather in one kernel over NVLink
        PeerExchangeArgs a{};
        a.rank = static_cast<uint32_t>(t->rank), a.world = static_cast<uint32_t>(t->world), a.shard = t->shard, a.n_params = t->n_params;
        a.n_mlp = kMlpParams, a.epoch = ++t->peer_epoch, a.lr = t->cfg.learning_rate, a.beta1 = 0.9f, a.beta2 = 0.99f, a.eps = 1e-15f;
        a.l2 = 1e-6f, a.loss_scale = kLossScale * static_cast<float>(t->world);
        a.grads  = reinterpret_cast<const __half* const*>(t->peer_table);
        a.params = reinterpret_cast<__half* const*>(t->peer_table + t->world);
        a.flags  = reinterpret_cast<uint32_t* const*>(t->peer_table + 2 * t->world);
        a.master = t->master, a.m = t->adam_m, a.v = t->adam_v, a.steps = t->adam_steps, a.lr_table = t->lr_table, a.table_len = t->lr_table_len;
        a.status = t->peer_status;
        NGP_TRY(peer_exchange_adam(a, t->stream));
    } else if (t->comm != nullptr) {
        const uint32_t first = static_cast<uint32_t>(t->rank) * t->shard;
        const uint32_t count = first < t->n_params ? std::min(t->shard, t->n_params - first) : 0u;
        NGP_TRY(ngp_adam_step_f16_range(count, first, kMlpParams, t->cfg.learning_rate, 0.9f, 0.99f, 1e-15f, 1e-6f,
                                        kLossScale * static_cast<float>(t->world), t->master + first, t->params + first, t->grads16 + first,
                                        t->adam_m + first, t->adam_v + first, t->adam_steps + first, t->lr_table, t->lr_table_len, t->stream));
        NGP_TRY(nccl_done(t, ncclAllGather(t->params + first, t->params, t->shard, ncclHalf, t->comm, t->stream), "ncclAllGather"));
    } else {
        NGP_TRY(ngp_adam_step_table(t->n_params, kMlpParams, t->cfg.learning_rate, 0.9f, 0.99f, 1e-15f, 1e-6f, kLossScale, t->master, t->params,
                                    t->grads, t->adam_m, t->adam_v, t->adam_steps, 1, t->lr_table, t->lr_table_len, t->stream));
    }
    mark(t, 8);
    if (t->profiling) {
        NGP_TRY(wait_stream(t, t->stream, "train step"));
        for (int k = 0; k < kTrainPhases; ++k) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, t->marks[k], t->marks[k + 1]);
            t->phase_ms[k] += ms;
        }
        t->inference_samples_sum += t->inference_samples;
        ++t->profiled_steps;
    }
    t->rays_per_batch    = next_rays;
    t->inference_samples = next_infer;
    t->step              = next_step;
    t->premarched        = premarch;
    return NGP_OK;
}

// One image (run_evaluation, ngp.train.cu:1597-1658): pixel rays in tiles of 2^18, each tile
// marched, evaluated and composited with one host read of its sample count.
int eval_image(ngp_trainer* t, const Split& s, uint32_t image, uint8_t* comparison_dev, float* rendered) {
    // A tile of `tile` pixels is marched; if its samples exceed the budget (MAX_SAMPLES) it is
    // re-marched in smaller tiles.  4096 pixels x 1024 steps always fit, as in the reference.
    const uint32_t total = s.width * s.height;
    uint32_t tile        = kNetworkBatch;
    for (uint32_t off = 0; off < total;) {
        const uint32_t n = std::min(tile, total - off);
        NGP_TRY(ngp_make_eval_rays(s.camera, image, s.width, s.height, s.fx, s.fy, s.cx, s.cy, off, n, t->rays, t->stream));
        NGP_TRY(ngp_march_rays(n, t->rays, 0, 0, t->bitfield, kMaxSamples, t->coords, t->numsteps, t->eval_march_scratch, t->counters + 1, t->stream));
        uint32_t used = 0;
        NGP_TRY(check_cuda(cudaMemcpyAsync(&used, t->counters + 1, sizeof(used), cudaMemcpyDeviceToHost, t->stream), "eval counter"));
        NGP_TRY(check_cuda(cudaStreamSynchronize(t->stream), "eval march"));
        if (used > kMaxSamples) {
            if (tile <= 4096u) return fail(NGP_ERR_OVERFLOW, "Evaluation sample budget overflowed (" + std::to_string(used) + " samples).");
            tile = std::max(4096u, tile / 4u);
            continue;
        }
        // network outputs only in front of each ray's stopping point (all the compositing reads)
        if (used > 0)
            NGP_TRY(ngp_eval_network_progressive(n, &t->layout, t->params, t->coords, used, t->numsteps, t->enc, used, t->out, t->rows, t->loss_scratch,
                                                 t->loss_scratch_bytes, t->stream));
        NGP_TRY(ngp_eval_composite(n, off, image, s.width, s.height, s.pixels, t->numsteps, t->coords, t->out, t->eval_sse, comparison_dev,
                                   rendered, t->stream));
        off += n;
    }
    return NGP_OK;
}

// One image by segmented marching: each tile's rays are marched a segment at a time (64 samples,
// then 128, then the rest), the network evaluated on the segment's samples, and the compositing
// continued; rays stop being marched once their transmittance falls below 1e-4.  Same samples,
// network outputs and compositing operations per pixel as eval_image, so the same image bit for
// bit; the march no longer runs through the (typically most) samples behind each ray's stopping
// point, and the tiles need no re-march when their samples exceed the budget.
// Tile set of a render: 64 x 64 tiles first, first + stride, ... (first = kAllPixels: every
// pixel in row-major order).
constexpr uint32_t kAllPixels = 0xFFFFFFFFu;

int eval_image_segmented(ngp_trainer* t, const Split& s, uint32_t image, uint8_t* comparison_dev, float* rendered, uint32_t first_tile = kAllPixels,
                         uint32_t tile_stride = 1u) {
    const bool tiled      = first_tile != kAllPixels;
    const uint32_t tiles_x = (s.width + 63u) / 64u, tiles_y = (s.height + 63u) / 64u;
    const uint32_t n_tiles = tiles_x * tiles_y;
    const uint32_t mine    = tiled ? (first_tile < n_tiles ? (n_tiles - first_tile + tile_stride - 1u) / tile_stride : 0u) : 0u;
    const uint32_t total   = tiled ? mine * 4096u : s.width * s.height;
    const cudaStream_t st  = t->stream;
    for (uint32_t off = 0; off < total; off += kSegTile) {
        const uint32_t n = std::min(kSegTile, total - off);
        if (tiled)
            NGP_TRY(ngp_make_eval_rays_tiles(s.camera, image, s.width, s.height, s.fx, s.fy, s.cx, s.cy, first_tile, tile_stride, off, n, t->rays, st));
        else
            NGP_TRY(ngp_make_eval_rays(s.camera, image, s.width, s.height, s.fx, s.fy, s.cx, s.cy, off, n, t->rays, st));
        uint32_t max_entries = n;
        for (uint32_t seg = 0;; ++seg) {
            const bool first         = seg == 0;
            const uint32_t* list     = first ? nullptr : t->seg_lists + static_cast<size_t>((seg - 1u) & 1u) * kSegTile;
            const uint32_t* n_dev    = first ? nullptr : t->seg_counters + 2u + ((seg - 1u) & 1u);
            const uint32_t cap       = kSegCaps[std::min<uint32_t>(seg, 2u)];
            NGP_TRY(ngp_march_rays_segment(max_entries, n_dev, list, t->rays, t->bitfield, first ? nullptr : t->seg_tstate,
                                           first ? nullptr : t->seg_marched, cap, kMaxSamples, t->coords, t->numsteps, t->seg_tout,
                                           t->eval_march_scratch, t->seg_counters, st));
            NGP_TRY(check_cuda(cudaMemcpyAsync(t->seg_host, t->seg_counters, 4 * sizeof(uint32_t), cudaMemcpyDeviceToHost, st), "segment counters"));
            NGP_TRY(check_cuda(cudaStreamSynchronize(st), "segment march"));
            const uint32_t complete = t->seg_host[1];
            if (complete == 0) break;  // no rays left in this tile
            const uint32_t used = std::min(t->seg_host[0], kMaxSamples);
            if (used > 0)
                NGP_TRY(ngp_eval_network_progressive(complete, &t->layout, t->params, t->coords, used, t->numsteps, t->enc, used, t->out, t->rows,
                                                     t->loss_scratch, t->loss_scratch_bytes, st));
            uint32_t* next_count = t->seg_counters + 2u + (seg & 1u);
            NGP_TRY(check_cuda(cudaMemsetAsync(next_count, 0, sizeof(uint32_t), st), "segment list count"));
            NGP_TRY(ngp_eval_composite_segment_tiles(max_entries, n_dev, t->seg_counters + 1, list, t->numsteps, t->coords, t->out, t->seg_tout,
                                                     t->seg_tstate, t->seg_marched, t->seg_state,
                                                     t->seg_lists + static_cast<size_t>(seg & 1u) * kSegTile, next_count, off, image, s.width,
                                                     s.height, s.pixels, t->eval_sse, comparison_dev, rendered, first_tile, tile_stride, st));
            // the next list holds at most this segment's entries
            if (!first) max_entries = t->seg_host[2u + ((seg - 1u) & 1u)];
        }
    }
    return NGP_OK;
}

int eval_one(ngp_trainer* t, const Split& s, uint32_t image, uint8_t* comparison_dev, float* rendered) {
    return t->eval_segmented ? eval_image_segmented(t, s, image, comparison_dev, rendered) : eval_image(t, s, image, comparison_dev, rendered);
}

int run_eval(ngp_trainer* t, const Split& s, uint32_t begin, uint32_t count, uint8_t* comparison_host, double* out_sse) {
    if (s.frames == 0) return fail(NGP_ERR_STATE, "no images in this split");
    if (begin >= s.frames || count > s.frames - begin) return fail(NGP_ERR_INVALID, "evaluation image range is out of bounds");
    if (comparison_host != nullptr) {
        if (count != 1) return fail(NGP_ERR_INVALID, "test comparison output requires exactly one image");
        cudaFree(t->comparison);
        NGP_TRY(dalloc(t->comparison, static_cast<size_t>(s.width) * s.height * 6u, "comparison image"));
    }
    NGP_TRY(check_cuda(cudaMemsetAsync(t->eval_sse, 0, sizeof(double), t->stream), "eval clear"));
    for (uint32_t k = 0; k < count; ++k) NGP_TRY(eval_one(t, s, begin + k, comparison_host != nullptr ? t->comparison : nullptr, nullptr));
    NGP_TRY(check_cuda(cudaMemcpyAsync(out_sse, t->eval_sse, sizeof(double), cudaMemcpyDeviceToHost, t->stream), "eval sse"));
    if (comparison_host != nullptr)
        NGP_TRY(check_cuda(cudaMemcpyAsync(comparison_host, t->comparison, static_cast<size_t>(s.width) * s.height * 6u, cudaMemcpyDeviceToHost,
                                           t->stream),
                           "comparison image"));
    return check_cuda(cudaStreamSynchronize(t->stream), "evaluation");
}

}  // namespace

extern "C" void ngp_trainer_default_config(ngp_trainer_config* cfg) {
    if (cfg == nullptr) return;
    *cfg                      = ngp_trainer_config{};
    cfg->n_levels             = 8;
    cfg->features_per_level   = 4;
    cfg->log2_hashmap_size    = 19;
    cfg->base_resolution      = 16;
    cfg->log2_per_level_scale = 1.0;
    cfg->learning_rate        = 1e-2f;
}

extern "C" int ngp_trainer_create(const ngp_trainer_config* cfg, const ngp_split* train, const ngp_split* validation, const ngp_split* test,
                                  ngp_trainer** out) {
    clear_error();
    if (out == nullptr || cfg == nullptr) return fail(NGP_ERR_INVALID, "trainer: null argument");
    *out = nullptr;
    if (train == nullptr || train->frame_count == 0) return fail(NGP_ERR_INVALID, "trainer: the training split is empty");
    if (cfg->n_levels * cfg->features_per_level != 32) return fail(NGP_ERR_INVALID, "trainer: the encoding must produce 32 features (levels x F)");
    auto* t      = new ngp_trainer{};
    t->cfg       = *cfg;
    if (const char* env = std::getenv("NGP_COLLECTIVE_TIMEOUT_MS"); env != nullptr && std::atof(env) > 0.0) t->collective_timeout_ms = std::atof(env);
    const int st = [&]() -> int {
        NGP_TRY(ngp_grid_layout_make(cfg->n_levels, cfg->features_per_level, cfg->log2_hashmap_size, cfg->base_resolution,
                                     cfg->log2_per_level_scale, &t->layout));
#if NGP_DP_PRIORITY
        // the training stream (with the gradient all-reduce) takes SM slots before the march
        int prio_low = 0, prio_high = 0;
        NGP_TRY(check_cuda(cudaDeviceGetStreamPriorityRange(&prio_low, &prio_high), "stream priorities"));
        NGP_TRY(check_cuda(cudaStreamCreateWithPriority(&t->stream, cudaStreamNonBlocking, prio_high), "stream"));
        NGP_TRY(check_cuda(cudaStreamCreateWithPriority(&t->march_stream, cudaStreamNonBlocking, prio_low), "march stream"));
#else
        NGP_TRY(check_cuda(cudaStreamCreateWithFlags(&t->stream, cudaStreamNonBlocking), "stream"));
        NGP_TRY(check_cuda(cudaStreamCreateWithFlags(&t->march_stream, cudaStreamNonBlocking), "march stream"));
#endif
        NGP_TRY(check_cuda(cudaEventCreateWithFlags(&t->ev_counts, cudaEventDisableTiming), "event"));
        NGP_TRY(check_cuda(cudaEventCreateWithFlags(&t->ev_march, cudaEventDisableTiming), "event"));
        NGP_TRY(check_cuda(cudaMallocHost(&t->host_counters, 8 * sizeof(uint32_t)), "pinned counters"));
        NGP_TRY(check_cuda(cudaMallocHost(&t->host_loss, kNetworkBatch * sizeof(float)), "pinned loss"));
        NGP_TRY(upload_split(t->train, train, "train"));
        NGP_TRY(upload_split(t->val, validation, "validation"));
        NGP_TRY(upload_split(t->test, test, "test"));
        t->n_params = kMlpParams + t->layout.n_params;
        NGP_TRY(dalloc(t->master, t->n_params, "params"));
        NGP_TRY(dalloc(t->params, t->n_params, "params fp16"));
        NGP_TRY(dalloc(t->grads, t->n_params, "gradients"));
        NGP_TRY(dalloc(t->grads16, t->n_params, "fp16 gradients"));
        NGP_TRY(dalloc(t->adam_m, t->n_params, "adam m"));
        NGP_TRY(dalloc(t->adam_v, t->n_params, "adam v"));
        NGP_TRY(dalloc(t->adam_steps, t->n_params, "adam steps"));
        NGP_TRY(dalloc(t->grid_values, kGridCells, "grid values"));
        NGP_TRY(dalloc(t->grid_scratch, kGridCells, "grid scratch"));
        NGP_TRY(dalloc(t->grid_partial, kGridCells / 1024u, "grid partial"));
        NGP_TRY(dalloc(t->grid_mean, 1, "grid mean"));
        NGP_TRY(dalloc(t->grid_indices, kGridCells, "grid indices"));
        NGP_TRY(dalloc(t->bitfield, kGridCells / 8u, "bitfield"));
        NGP_TRY(dalloc(t->occupied, 1, "occupied count"));
        NGP_TRY(dalloc(t->grid_counter, 1, "grid sample counter"));
        for (MarchSet& m : t->sets) {
            NGP_TRY(dalloc(m.coords, static_cast<size_t>(kMaxSamples) * 7u, "sample coords"));
            NGP_TRY(dalloc(m.rays, static_cast<size_t>(kNetworkBatch) * 6u, "rays"));
            NGP_TRY(dalloc(m.ray_indices, kNetworkBatch, "ray indices"));
            NGP_TRY(dalloc(m.numsteps, static_cast<size_t>(kNetworkBatch) * 2u, "numsteps"));
            NGP_TRY(dalloc(m.counters, 8, "counters"));
            NGP_TRY(check_cuda(cudaMemsetAsync(m.counters, 0, 8 * sizeof(uint32_t), t->stream), "clear counters"));
            NGP_TRY(check_cuda(cudaMemsetAsync(m.coords, 0, sizeof(float) * kMaxSamples * 7u, t->stream), "clear coords"));
        }
        t->coords = t->sets[2].coords, t->rays = t->sets[2].rays, t->ray_indices = t->sets[2].ray_indices;
        t->numsteps = t->sets[2].numsteps, t->counters = t->sets[2].counters;
        NGP_TRY(dalloc(t->eval_march_scratch, ngp_march_scratch_words(kNetworkBatch), "evaluation march scratch"));
        NGP_TRY(dalloc(t->march_scratch, ngp_march_scratch_words(kNetworkBatch), "march scratch"));
        NGP_TRY(dalloc(t->enc, static_cast<size_t>(kMaxSamples) * 32u, "encoded positions"));
        NGP_TRY(dalloc(t->out, static_cast<size_t>(kMaxSamples) * 16u, "network output"));
        NGP_TRY(dalloc(t->rows, kMaxSamples, "row list"));
        NGP_TRY(dalloc(t->batch_rows, kCompactedRows, "batch rows"));
        // a batch that selects nothing still reads valid (zero) rows before the step reports it
        NGP_TRY(check_cuda(cudaMemsetAsync(t->batch_rows, 0, sizeof(uint32_t) * kCompactedRows, t->stream), "clear batch rows"));
        NGP_TRY(dalloc(t->dens, kMaxSamples, "densities"));
        NGP_TRY(dalloc(t->grid_density, kGridCells, "grid density"));
        NGP_TRY(dalloc(t->ccoords, static_cast<size_t>(kCompactedRows) * 7u, "compacted coords"));
        NGP_TRY(dalloc(t->cout, static_cast<size_t>(kCompactedRows) * 16u, "compacted network output"));
        NGP_TRY(dalloc(t->dloss, static_cast<size_t>(kNetworkBatch) * 16u, "output gradients"));
        NGP_TRY(dalloc(t->loss_values, kNetworkBatch, "loss values"));
        t->loss_scratch_bytes = ngp_loss_scratch_bytes(kNetworkBatch);
        NGP_TRY(dalloc(t->loss_scratch, t->loss_scratch_bytes, "loss scratch"));
        NGP_TRY(dalloc(t->cenc, static_cast<size_t>(kCompactedRows) * 32u, "batch encoding"));
        NGP_TRY(dalloc(t->denc, static_cast<size_t>(kNetworkBatch) * 32u, "encoding gradient"));
        t->mlp_scratch_floats = ngp_mlp_backward_scratch_floats();
        NGP_TRY(dalloc(t->mlp_scratch, t->mlp_scratch_floats, "mlp scratch"));
        NGP_TRY(dalloc(t->eval_sse, 1, "eval sse"));
        NGP_TRY(dalloc(t->seg_tout, kSegTile, "segment t"));
        NGP_TRY(dalloc(t->seg_tstate, kSegTile, "segment ray t"));
        NGP_TRY(dalloc(t->seg_marched, kSegTile, "segment ray counts"));
        NGP_TRY(dalloc(t->seg_state, static_cast<size_t>(kSegTile) * 4u, "segment ray state"));
        NGP_TRY(dalloc(t->seg_lists, static_cast<size_t>(kSegTile) * 2u, "segment lists"));
        NGP_TRY(dalloc(t->seg_counters, 4, "segment counters"));
        NGP_TRY(check_cuda(cudaMallocHost(&t->seg_host, 4 * sizeof(uint32_t)), "segment host counters"));
        NGP_TRY(dalloc(t->lr_table, kLrTableCapacity, "adam rate table"));
        const cudaStream_t s = t->stream;
        NGP_TRY(check_cuda(cudaMemsetAsync(t->grads, 0, sizeof(float) * t->n_params, s), "clear grads"));
        NGP_TRY(check_cuda(cudaMemsetAsync(t->adam_m, 0, sizeof(float) * t->n_params, s), "clear m"));
        NGP_TRY(check_cuda(cudaMemsetAsync(t->adam_v, 0, sizeof(float) * t->n_params, s), "clear v"));
        NGP_TRY(check_cuda(cudaMemsetAsync(t->adam_steps, 0, sizeof(uint32_t) * t->n_params, s), "clear steps"));
        NGP_TRY(check_cuda(cudaMemsetAsync(t->grid_values, 0, sizeof(float) * kGridCells, s), "clear grid"));
        NGP_TRY(check_cuda(cudaMemsetAsync(t->grid_scratch, 0, sizeof(float) * kGridCells, s), "clear scratch"));
        NGP_TRY(check_cuda(cudaMemsetAsync(t->bitfield, 0xFF, kGridCells / 8u, s), "fill bitfield"));
        NGP_TRY(init_params(t));
        return check_cuda(cudaStreamSynchronize(s), "trainer init");
    }();
    if (st != NGP_OK) {
        destroy(t);
        return st;
    }
    *out = t;
    return NGP_OK;
}

extern "C" void ngp_trainer_destroy(ngp_trainer* t) { destroy(t); }

extern "C" int ngp_nccl_unique_id(uint8_t* out, size_t bytes) {
    clear_error();
    if (out == nullptr || bytes < sizeof(ncclUniqueId)) return fail(NGP_ERR_INVALID, "nccl id: buffer too small");
    ncclUniqueId id;
    const ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return fail(NGP_ERR_CUDA, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
    std::memcpy(out, &id, sizeof(id));
    return NGP_OK;
}

namespace {
// Maps every rank's fp16 gradient, fp16 parameter and flag buffers into this process (CUDA IPC;
// the handles travel through an NCCL all-gather) and enables the fused exchange when every rank
// succeeded (an NCCL min-reduction of the ranks' outcomes).  Otherwise the mappings are closed
// and the NCCL path stays in use.
int setup_peer_exchange(ngp_trainer* t) {
    const int W = t->world;
    NGP_TRY(dalloc(t->peer_flags, 2u * static_cast<uint32_t>(W) + 1u, "peer flags"));
    NGP_TRY(dalloc(t->peer_status, 1, "peer exchange status"));
    NGP_TRY(check_cuda(cudaMemset(t->peer_flags, 0, sizeof(uint32_t) * (2u * W + 1u)), "peer flags"));
    NGP_TRY(check_cuda(cudaMemset(t->peer_status, 0, sizeof(uint32_t)), "peer status"));
    constexpr size_t kH = sizeof(cudaIpcMemHandle_t);
    std::vector<unsigned char> mine(3 * kH), all(static_cast<size_t>(W) * 3 * kH);
    int ok = 1;
    void* bufs[3] = {t->grads16, t->params, t->peer_flags};
    for (int k = 0; k < 3; ++k) {
        cudaIpcMemHandle_t h{};
        if (cudaIpcGetMemHandle(&h, bufs[k]) != cudaSuccess) ok = 0;
        std::memcpy(mine.data() + k * kH, &h, kH);
    }
    (void)cudaGetLastError();
    unsigned char* dev = nullptr;
    NGP_TRY(dalloc(dev, all.size() + 16, "peer handles"));
    int st = check_cuda(cudaMemcpy(dev + static_cast<size_t>(t->rank) * 3 * kH, mine.data(), mine.size(), cudaMemcpyHostToDevice), "peer handles");
    if (st == NGP_OK)
        st = nccl_done(t, ncclAllGather(dev + static_cast<size_t>(t->rank) * 3 * kH, dev, 3 * kH, ncclUint8, t->comm, t->stream), "ncclAllGather handles");
    if (st == NGP_OK) st = wait_stream(t, t->stream, "peer handles");
    if (st == NGP_OK) st = check_cuda(cudaMemcpy(all.data(), dev, all.size(), cudaMemcpyDeviceToHost), "peer handles");
    if (st != NGP_OK) {
        cudaFree(dev);
        return st;
    }
    std::vector<void*> table(3 * static_cast<size_t>(W), nullptr);
    for (int q = 0; q < W; ++q)
        for (int k = 0; k < 3; ++k) {
            if (q == t->rank) {
                table[k * W + q] = bufs[k];
                continue;
            }
            cudaIpcMemHandle_t h{};
            std::memcpy(&h, all.data() + (static_cast<size_t>(q) * 3 + k) * kH, kH);
            void* p = nullptr;
            if (ok && cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess) {
                table[k * W + q] = p;
                t->peer_opened.push_back(p);
            } else {
                ok = 0;
            }
        }
    (void)cudaGetLastError();
    // every rank must be able to use the fused path
    int* agree = reinterpret_cast<int*>(dev + all.size());
    st = check_cuda(cudaMemcpy(agree, &ok, sizeof(int), cudaMemcpyHostToDevice), "peer agreement");
    if (st == NGP_OK) st = nccl_done(t, ncclAllReduce(agree, agree, 1, ncclInt32, ncclMin, t->comm, t->stream), "ncclAllReduce agreement");
    if (st == NGP_OK) st = wait_stream(t, t->stream, "peer agreement");
    if (st == NGP_OK) st = check_cuda(cudaMemcpy(&ok, agree, sizeof(int), cudaMemcpyDeviceToHost), "peer agreement");
    cudaFree(dev);
    NGP_TRY(st);
    if (!ok) {
        for (void* q : t->peer_opened) cudaIpcCloseMemHandle(q);
        t->peer_opened.clear();
        return NGP_OK;
    }
    NGP_TRY(dalloc(t->peer_table, table.size(), "peer table"));
    NGP_TRY(check_cuda(cudaMemcpy(t->peer_table, table.data(), sizeof(void*) * table.size(), cudaMemcpyHostToDevice), "peer table"));
    t->peer_exchange = true;
    return NGP_OK;
}
}  // namespace

extern "C" int ngp_trainer_join(ngp_trainer* t, const uint8_t* unique_id, int world, int rank) {
    clear_error();
    if (t == nullptr || unique_id == nullptr || world < 1 || rank < 0 || rank >= world) return fail(NGP_ERR_INVALID, "trainer join: bad arguments");
    if (t->step != 0) return fail(NGP_ERR_STATE, "trainer join: only before training");
    if (t->comm != nullptr) return fail(NGP_ERR_STATE, "trainer join: already joined");
    if (world == 1) return NGP_OK;
    // padded exchange buffers: the fp16 parameters and gradients hold n_padded entries so that
    // every rank's shard has the same length (a multiple of 8: the exchange kernel moves 16-byte
    // groups of fp16 values)
    const uint64_t unit   = 8ull * static_cast<uint64_t>(world);
    const uint64_t padded = (static_cast<uint64_t>(t->n_params) + unit - 1u) / unit * unit;
    if (padded > 0xFFFFFFFFull) return fail(NGP_ERR_INVALID, "trainer join: too many parameters for the exchange");
    uint16_t *params = nullptr, *grads16 = nullptr;
    NGP_TRY(dalloc(params, padded, "padded fp16 params"));
    if (const int st = dalloc(grads16, padded, "padded fp16 gradients"); st != NGP_OK) {
        cudaFree(params);
        return st;
    }
    cudaMemsetAsync(params, 0, padded * sizeof(uint16_t), t->stream);
    cudaMemsetAsync(grads16, 0, padded * sizeof(uint16_t), t->stream);
    cudaMemcpyAsync(params, t->params, sizeof(uint16_t) * t->n_params, cudaMemcpyDeviceToDevice, t->stream);
    if (const int st = check_cuda(cudaStreamSynchronize(t->stream), "trainer join: padded buffers"); st != NGP_OK) {
        cudaFree(params), cudaFree(grads16);
        return st;
    }
    cudaFree(t->params), cudaFree(t->grads16);
    t->params   = params;
    t->grads16  = grads16;
    t->n_padded = static_cast<uint32_t>(padded);
    t->shard    = static_cast<uint32_t>(padded / static_cast<uint64_t>(world));
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking     = 0;
    ncclComm_t comm     = nullptr;
    const ncclResult_t r = ncclCommInitRankConfig(&comm, world, id, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress) return fail(NGP_ERR_CUDA, std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
    t->comm  = comm;
    t->world = world;
    t->rank  = rank;
    const int st = wait_comm(t, [&]() -> int {
        ncclResult_t a = ncclSuccess;
        ncclCommGetAsyncError(t->comm, &a);
        if (a == ncclSuccess) return 1;
        if (a == ncclInProgress) return 0;
        set_error(ncclGetErrorString(a));
        return -1;
    }, "ncclCommInitRankConfig");
    if (st != NGP_OK) {
        t->world = 1, t->rank = 0;
        return st;
    }
    const char* mode = std::getenv("NGP_EXCHANGE");
    if (mode == nullptr || std::string(mode) != "nccl") NGP_TRY(setup_peer_exchange(t));
    return NGP_OK;
}

extern "C" int ngp_trainer_set_loss(ngp_trainer* t, int loss_kind) {
    clear_error();
    if (t == nullptr || (loss_kind != 0 && loss_kind != 1)) return fail(NGP_ERR_INVALID, "set loss: bad arguments (0 = L2, 1 = Huber)");
    t->loss_kind = loss_kind;
    return NGP_OK;
}

extern "C" int ngp_trainer_exchange_mode(const ngp_trainer* t) {
    if (t == nullptr || t->comm == nullptr) return 0;
    return t->peer_exchange ? 2 : 1;
}

extern "C" int ngp_trainer_set_collective_timeout(ngp_trainer* t, double timeout_ms) {
    clear_error();
    if (t == nullptr || !(timeout_ms > 0.0)) return fail(NGP_ERR_INVALID, "collective timeout: bad arguments");
    t->collective_timeout_ms = timeout_ms;
    return NGP_OK;
}

extern "C" int ngp_trainer_train(ngp_trainer* t, int32_t iters, ngp_train_stats* stats) {
    clear_error();
    if (t == nullptr) return fail(NGP_ERR_INVALID, "trainer is null");
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, t->stream);
    t->grid_update_ms  = 0.0f;
    uint32_t loss_rays = t->rays_per_batch;
    for (int32_t i = 0; i < iters; ++i) {
        loss_rays    = t->rays_per_batch;
        // the last step also marches the next one: it is consumed by the next train call
        const int st = train_step(t, true);
        if (st != NGP_OK) {
            cudaStreamSynchronize(t->march_stream);
            t->premarched = false;
            cudaEventDestroy(e0);
            cudaEventDestroy(e1);
            return st;
        }
    }
    cudaEventRecord(e1, t->stream);
    NGP_TRY(check_cuda(cudaMemcpyAsync(t->host_loss, t->loss_values, sizeof(float) * loss_rays, cudaMemcpyDeviceToHost, t->stream), "read loss"));
    NGP_TRY(check_cuda(cudaMemcpyAsync(&t->occupied_cells, t->occupied, sizeof(uint32_t), cudaMemcpyDeviceToHost, t->stream), "read occupied"));
    cudaEvent_t e2 = nullptr;
    NGP_TRY(check_cuda(cudaEventCreateWithFlags(&e2, cudaEventDisableTiming), "train event"));
    cudaEventRecord(e2, t->stream);
    // the next step's grid-update first half runs while the host returns (it is not waited for)
    const int begun = begin_next_grid_update(t);
    const int waited = wait_event(t, e2, "train");
    cudaEventDestroy(e2);
    NGP_TRY(begun);
    NGP_TRY(waited);
    if (t->peer_exchange) {
        uint32_t status = 0;
        NGP_TRY(check_cuda(cudaMemcpy(&status, t->peer_status, sizeof(status), cudaMemcpyDeviceToHost), "peer exchange status"));
        if (status != 0)
            return abort_comm(t, NGP_ERR_TIMEOUT, "peer exchange: a rank did not arrive within 2 s (status " + std::to_string(status) +
                                                      "); communicator aborted");
    }
    collect_grid_times(t);
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    float loss_sum = 0.0f;
    for (uint32_t r = 0; r < loss_rays; ++r) loss_sum += t->host_loss[r];
    if (stats != nullptr) {
        stats->step                                    = t->step;
        stats->rays_per_batch                          = t->rays_per_batch;
        stats->measured_sample_count_before_compaction = t->measured_before;
        stats->measured_sample_count                   = t->measured;
        stats->density_grid_occupied_cells             = t->occupied_cells;
        stats->loss                                    = loss_sum * static_cast<float>(t->measured) / static_cast<float>(kNetworkBatch);
        stats->elapsed_ms                              = ms;
        stats->density_grid_update_ms                  = t->grid_update_ms;
        stats->density_grid_occupancy_ratio            = static_cast<float>(t->occupied_cells) / static_cast<float>(kGridCells);
    }
    return NGP_OK;
}

extern "C" int ngp_trainer_evaluate(ngp_trainer* t, int split, uint32_t image_begin, uint32_t image_count, uint8_t* comparison_host,
                                    double* out_sse, uint64_t* out_pixels) {
    clear_error();
    if (t == nullptr || out_sse == nullptr) return fail(NGP_ERR_INVALID, "evaluate: null argument");
    const Split& s = split == 1 ? t->val : t->test;
    NGP_TRY(run_eval(t, s, image_begin, image_count, comparison_host, out_sse));
    if (out_pixels != nullptr) *out_pixels = static_cast<uint64_t>(s.width) * s.height * image_count;
    return NGP_OK;
}

extern "C" int ngp_trainer_render(ngp_trainer* t, const float* camera_host, uint32_t width, uint32_t height, float fx, float fy, float cx,
                                  float cy, float* rgb_device) {
    clear_error();
    if (t == nullptr || camera_host == nullptr || rgb_device == nullptr || width == 0 || height == 0 || !(fx > 0) || !(fy > 0))
        return fail(NGP_ERR_INVALID, "render: bad input");
    Split s{};
    s.frames = 1, s.width = width, s.height = height, s.fx = fx, s.fy = fy, s.cx = cx, s.cy = cy;
    NGP_TRY(dalloc(s.camera, 12, "render camera"));
    int st = check_cuda(cudaMemcpyAsync(s.camera, camera_host, sizeof(float) * 12u, cudaMemcpyHostToDevice, t->stream), "render camera");
    if (st == NGP_OK) st = eval_one(t, s, 0, nullptr, rgb_device);
    if (st == NGP_OK) st = check_cuda(cudaStreamSynchronize(t->stream), "render");
    free_split(s);
    return st;
}

extern "C" int ngp_trainer_render_tiles(ngp_trainer* t, const float* camera_host, uint32_t width, uint32_t height, float fx, float fy, float cx,
                                        float cy, uint32_t first_tile, uint32_t tile_stride, float* rgb_device) {
    clear_error();
    if (t == nullptr || camera_host == nullptr || rgb_device == nullptr || width == 0 || height == 0 || !(fx > 0) || !(fy > 0) || tile_stride == 0)
        return fail(NGP_ERR_INVALID, "render tiles: bad input");
    Split s{};
    s.frames = 1, s.width = width, s.height = height, s.fx = fx, s.fy = fy, s.cx = cx, s.cy = cy;
    NGP_TRY(dalloc(s.camera, 12, "render camera"));
    int st = check_cuda(cudaMemcpyAsync(s.camera, camera_host, sizeof(float) * 12u, cudaMemcpyHostToDevice, t->stream), "render camera");
    if (st == NGP_OK) st = eval_image_segmented(t, s, 0, nullptr, rgb_device, first_tile, tile_stride);
    if (st == NGP_OK) st = check_cuda(cudaStreamSynchronize(t->stream), "render");
    free_split(s);
    return st;
}

extern "C" void ngp_adaptive_batch(uint32_t rays_per_batch, uint32_t measured_before, uint32_t measured, uint32_t* next_rays,
                                   uint32_t* next_inference_samples) {
    const uint32_t g = kBatchGranule;
    *next_inference_samples = ((std::min(measured_before, kMaxSamples) + g - 1u) / g) * g;
    if (measured == 0u) {  // no step follows (the trainer stops); keep the batch
        *next_rays = rays_per_batch;
        return;
    }
    const uint64_t want = std::min<uint64_t>((static_cast<uint64_t>(rays_per_batch) * kNetworkBatch) / measured, kNetworkBatch);
    *next_rays          = std::min(std::max(static_cast<uint32_t>((want + g - 1u) / g * g), g), kNetworkBatch);
}

extern "C" int ngp_trainer_set_segmented_eval(ngp_trainer* t, int enabled) {
    clear_error();
    if (t == nullptr) return fail(NGP_ERR_INVALID, "segmented eval: null trainer");
    t->eval_segmented = enabled != 0;
    return NGP_OK;
}

extern "C" uint32_t ngp_trainer_param_count(const ngp_trainer* t) { return t == nullptr ? 0u : t->n_params; }

extern "C" int ngp_trainer_get_params(ngp_trainer* t, float* host_out, uint32_t count) {
    clear_error();
    if (t == nullptr || host_out == nullptr || count != t->n_params) return fail(NGP_ERR_INVALID, "get params: bad arguments");
    if (t->comm == nullptr) return check_cuda(cudaMemcpy(host_out, t->master, sizeof(float) * count, cudaMemcpyDeviceToHost), "download params");
    // data parallel: each rank's fp32 master is current only on its own shard; the shards are
    // all-gathered into a temporary buffer (a collective: every rank calls this)
    float* full = nullptr;
    NGP_TRY(dalloc(full, t->n_padded, "gathered params"));
    const size_t first = static_cast<size_t>(t->rank) * t->shard;
    const size_t mine  = first < t->n_params ? std::min<size_t>(t->shard, t->n_params - first) : 0;
    int st             = check_cuda(cudaMemsetAsync(full, 0, sizeof(float) * t->n_padded, t->stream), "gather params");
    if (st == NGP_OK && mine > 0) st = check_cuda(cudaMemcpyAsync(full + first, t->master + first, sizeof(float) * mine, cudaMemcpyDeviceToDevice, t->stream), "gather params");
    if (st == NGP_OK) st = nccl_done(t, ncclAllGather(full + first, full, t->shard, ncclFloat32, t->comm, t->stream), "ncclAllGather params");
    if (st == NGP_OK) st = wait_stream(t, t->stream, "gather params");
    if (st == NGP_OK) st = check_cuda(cudaMemcpy(host_out, full, sizeof(float) * count, cudaMemcpyDeviceToHost), "download params");
    cudaFree(full);
    return st;
}

extern "C" int ngp_trainer_set_params(ngp_trainer* t, const float* host_in, uint32_t count) {
    clear_error();
    if (t == nullptr || host_in == nullptr || count != t->n_params) return fail(NGP_ERR_INVALID, "set params: bad arguments");
    if (t->step != 0) return fail(NGP_ERR_STATE, "weights can only be loaded before training");
    NGP_TRY(check_cuda(cudaMemcpy(t->master, host_in, sizeof(float) * count, cudaMemcpyHostToDevice), "upload params"));
    NGP_TRY(check_cuda(cudaMemset(t->grads, 0, sizeof(float) * count), "clear grads"));
    NGP_TRY(check_cuda(cudaMemset(t->adam_m, 0, sizeof(float) * count), "clear m"));
    NGP_TRY(check_cuda(cudaMemset(t->adam_v, 0, sizeof(float) * count), "clear v"));
    NGP_TRY(check_cuda(cudaMemset(t->adam_steps, 0, sizeof(uint32_t) * count), "clear steps"));
    cast_half_kernel<<<(count + 255) / 256, 256, 0, t->stream>>>(t->master, reinterpret_cast<__half*>(t->params), count);
    NGP_TRY(check_launch("cast_half_kernel"));
    return check_cuda(cudaStreamSynchronize(t->stream), "set params");
}

extern "C" int ngp_trainer_get_grid(const ngp_trainer* t, uint8_t* bitfield_host, float* values_host) {
    clear_error();
    if (t == nullptr) return fail(NGP_ERR_INVALID, "get grid: null trainer");
    if (bitfield_host != nullptr) NGP_TRY(check_cuda(cudaMemcpy(bitfield_host, t->bitfield, kGridCells / 8u, cudaMemcpyDeviceToHost), "bitfield"));
    if (values_host != nullptr) NGP_TRY(check_cuda(cudaMemcpy(values_host, t->grid_values, sizeof(float) * kGridCells, cudaMemcpyDeviceToHost), "values"));
    return NGP_OK;
}

extern "C" int ngp_trainer_set_run_ahead(ngp_trainer* t, int enable) {
    clear_error();
    if (t == nullptr) return fail(NGP_ERR_INVALID, "run ahead: null trainer");
    t->run_ahead = enable != 0;
    return enable ? NGP_OK : discard_grid_begin(t);
}

extern "C" int ngp_trainer_set_profiling(ngp_trainer* t, int enable) {
    clear_error();
    if (t == nullptr) return fail(NGP_ERR_INVALID, "profiling: null trainer");
    if (enable && t->marks[0] == nullptr) {
        for (cudaEvent_t& e : t->marks) NGP_TRY(check_cuda(cudaEventCreate(&e), "profiling events"));
        for (cudaEvent_t& e : t->grid_marks) NGP_TRY(check_cuda(cudaEventCreate(&e), "profiling events"));
    }
    if (enable) NGP_TRY(discard_grid_begin(t));  // profiled updates are timed whole
    t->profiling = enable != 0;
    for (double& v : t->phase_ms) v = 0.0;
    for (double& v : t->grid_phase_ms) v = 0.0;
    t->inference_samples_sum = 0.0;
    t->profiled_steps        = 0;
    t->grid_samples_sum      = 0.0;
    t->profiled_grid_updates = 0;
    return NGP_OK;
}

extern "C" int ngp_trainer_grid_phase_times(const ngp_trainer* t, float* out_ms, uint32_t n, uint32_t* out_updates, float* out_mean_samples) {
    clear_error();
    if (t == nullptr || out_ms == nullptr || n < static_cast<uint32_t>(kGridPhases)) return fail(NGP_ERR_INVALID, "grid phase times: bad arguments");
    for (int k = 0; k < kGridPhases; ++k) out_ms[k] = static_cast<float>(t->grid_phase_ms[k]);
    if (out_updates != nullptr) *out_updates = t->profiled_grid_updates;
    if (out_mean_samples != nullptr)
        *out_mean_samples = t->profiled_grid_updates ? static_cast<float>(t->grid_samples_sum / t->profiled_grid_updates) : 0.0f;
    return NGP_OK;
}

extern "C" int ngp_trainer_phase_times(const ngp_trainer* t, float* out_ms, uint32_t n, uint32_t* out_steps, float* out_mean_inference_samples) {
    clear_error();
    if (t == nullptr || out_ms == nullptr || n < static_cast<uint32_t>(kTrainPhases)) return fail(NGP_ERR_INVALID, "phase times: bad arguments");
    for (int k = 0; k < kTrainPhases; ++k) out_ms[k] = static_cast<float>(t->phase_ms[k]);
    if (out_steps != nullptr) *out_steps = t->profiled_steps;
    if (out_mean_inference_samples != nullptr)
        *out_mean_inference_samples = t->profiled_steps ? static_cast<float>(t->inference_samples_sum / t->profiled_steps) : 0.0f;
    return NGP_OK;
}

// initialize_mlp_parameters (ngp.train.cu:1423-1461): Xavier-uniform per matrix from one PCG32
// stream (seed 1337) in the packed order, fp32 master + fp16 copy.
extern "C" int ngp_init_mlp_parameters(float* master, uint16_t* params, void* stream) {
    clear_error();
    if (master == nullptr || params == nullptr) return fail(NGP_ERR_INVALID, "init mlp parameters: null pointer");
    std::vector<float> h(kMlpParams);
    Pcg32 rng{kTrainSeed};
    const uint32_t shapes[5][2] = {{64, 32}, {16, 64}, {64, 32}, {64, 64}, {16, 64}};
    uint32_t off                = 0;
    for (auto& sh : shapes) {
        const float scale = std::sqrt(6.0f / static_cast<float>(sh[0] + sh[1]));
        for (uint32_t i = 0; i < sh[0] * sh[1]; ++i) h[off + i] = rng.next_float() * 2.0f * scale - scale;
        off += sh[0] * sh[1];
    }
    const cudaStream_t s = as_stream(stream);
    NGP_TRY(check_cuda(cudaMemcpyAsync(master, h.data(), sizeof(float) * kMlpParams, cudaMemcpyHostToDevice, s), "upload mlp params"));
    cast_half_kernel<<<(kMlpParams + 255) / 256, 256, 0, s>>>(master, reinterpret_cast<__half*>(params), kMlpParams);
    NGP_TRY(check_launch("cast_half_kernel"));
    return check_cuda(cudaStreamSynchronize(s), "init mlp parameters");  // h goes out of scope
}

// initialize_grid_params_kernel (ngp.train.cu:1002-1017): U(-1e-4, 1e-4) from the PCG32 stream
// continued after the MLP's draws, four values per thread.
extern "C" int ngp_init_grid_parameters(uint32_t n_grid, float* master_grid, uint16_t* params_grid, void* stream) {
    clear_error();
    if (n_grid == 0) return NGP_OK;
    if (master_grid == nullptr || params_grid == nullptr) return fail(NGP_ERR_INVALID, "init grid parameters: null pointer");
    const uint32_t n_threads = (n_grid + 3u) / 4u;
    init_grid_kernel<<<(n_threads + 127u) / 128u, 128, 0, as_stream(stream)>>>(master_grid, reinterpret_cast<__half*>(params_grid), n_grid, kMlpParams);
    return check_launch("init_grid_kernel");
}

extern "C" int ngp_cast_to_half(uint32_t n, const float* in, uint16_t* out, void* stream) {
    clear_error();
    if (n == 0) return NGP_OK;
    if (in == nullptr || out == nullptr) return fail(NGP_ERR_INVALID, "cast to half: null pointer");
    cast_half_kernel<<<(n + 255u) / 256u, 256, 0, as_stream(stream)>>>(in, reinterpret_cast<__half*>(out), n);
    return check_launch("cast_half_kernel");
}
