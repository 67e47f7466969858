// Fully fused 64-wide density + colour MLPs on the sm_100a tensor cores (tcgen05 + TMEM).
//
// Replaces the reference's WMMA kernels and cuBLASLt GEMMs (ngp.train.cu:1019-1236,
// 1494-1524, 1660-1903):
//   density net  32 -> 64 (ReLU) -> 16           (output 0 = raw density)
//   colour net   [16 density outputs | 16 SH] -> 64 (ReLU) -> 64 (ReLU) -> 16 (0-2 = raw rgb)
// fp16 weights [out][in] packed as in ngp.train.h:58-78, no biases, fp32 accumulation in TMEM,
// one fp16 rounding per layer output.
//
// Execution: a persistent CTA of one warpgroup (128 threads) owns a 128-row tile at a time;
// thread t owns row t, which is TMEM lane t of every accumulator.  All weights stay in shared
// memory for the CTA's lifetime; activations never leave the SM: each layer's accumulator is
// read from TMEM (tcgen05.ld), activated, rounded to fp16 and written back into shared memory
// as the next MMA's operand.  One elected thread issues the MMAs and commits them to an
// mbarrier that every thread waits on (with a time bound).
//
// Backward recomputes the forward activations of its tile on chip instead of reading stored
// hidden activations from HBM, then runs the input-gradient chain and accumulates all five
// weight gradients in TMEM across every tile the CTA processes.  Each CTA writes its weight-
// gradient partial once; a second small kernel sums the partials in a fixed order
// (deterministic).  Weight-gradient GEMMs use M = 128 with the 64 real rows in lanes 0-63.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "sampler.cuh"
#include "umma.cuh"

namespace ngp {
namespace {

constexpr uint32_t kThreads = 128;
constexpr uint32_t kRows    = 128;

// packed weight offsets (halves)
constexpr uint32_t kWdIn = 0, kWdOut = 2048, kWrIn = 3072, kWrH = 5120, kWrOut = 9216, kMlpParams = 10240;

// shared-memory weight tiles (bytes): each [out rows][in] in the interleaved layout
constexpr uint32_t kSWdIn = 0, kSWdOut = 4096, kSWrIn = 6144, kSWrH = 10240, kSWrOut = 18432, kSWeights = 20480;

// ---- error status --------------------------------------------------------------------------
// Device status word: set (never cleared by kernels) when an mbarrier wait times out.
__device__ uint32_t g_mlp_status;

#ifdef NGP_MLP_TRACE
// Development-only timeline of CTA 0 of the last forward launch (SM clock at fixed points).
__device__ unsigned long long g_mlp_trace[64];
#define MLP_TRACE(i) do { if (blockIdx.x == 0 && threadIdx.x == 0 && ((i) < 60 || (i) == 63)) g_mlp_trace[(i)] = clock64(); } while (0)
extern "C" __attribute__((visibility("default"))) int ngp_mlp_trace_read(unsigned long long* out) {
    return static_cast<int>(cudaMemcpyFromSymbol(out, g_mlp_trace, sizeof(g_mlp_trace)));
}
#else
#define MLP_TRACE(i) do { } while (0)
#endif

// ---- tile helpers --------------------------------------------------------------------------
// Byte offset of 16-byte chunk c of row r in a tile with `cpr` chunks per row.
__device__ __forceinline__ uint32_t tile_off(uint32_t r, uint32_t c, uint32_t cpr) { return (r & 7u) * 16u + (r >> 3) * (128u * cpr) + c * 128u; }

__device__ __forceinline__ void store_chunk(unsigned char* tile, uint32_t r, uint32_t c, uint32_t cpr, uint4 v) {
    *reinterpret_cast<uint4*>(tile + tile_off(r, c, cpr)) = v;
}
__device__ __forceinline__ uint4 load_chunk(const unsigned char* tile, uint32_t r, uint32_t c, uint32_t cpr) {
    return *reinterpret_cast<const uint4*>(tile + tile_off(r, c, cpr));
}

// Asynchronous 16-byte global -> shared copy (cp.async, L2 only); src_bytes = 0 zero-fills.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(umma::smem_addr(smem_dst)), "l"(gsrc), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Row-major encoded inputs ([rows][32] fp16, NGP_ROWS): tile row r's 64 bytes arrive as four
// 16-byte asynchronous copies straight into the interleaved operand tile (chunk c of row r at
// tile_off(r, c, 4)); rows past the end are zero-filled.  One commit group per call.
__device__ __forceinline__ void issue_row_copy(unsigned char* tile, uint32_t r, const __half* x, uint32_t col, bool valid) {
    const __half* src = x + static_cast<uint64_t>(valid ? col : 0u) * 32u;
#pragma unroll
    for (uint32_t c = 0; c < 4; ++c) cp_async16(tile + tile_off(r, c, 4), src + c * 8u, valid ? 16u : 0u);
    cp_async_commit();
}

// Feature-major inputs of contiguous rows ([32][x_stride] fp16, no row list): feature k of the
// tile's rows r0 .. r0 + 127 is one 256-byte run, copied as 16 chunks of 16 bytes into the
// tile as the MN-major A operand (tile row k, the 128 rows along it: chunk (k, c) at
// tile_off(k, c, 16)); rows past n are zero-filled.  Four copies per thread, one commit group.
__device__ __forceinline__ void issue_col_copy(unsigned char* tile, const __half* x, uint32_t x_stride, uint32_t r0, uint32_t n) {
#pragma unroll
    for (uint32_t j = 0; j < 4; ++j) {
        const uint32_t q = threadIdx.x + j * 128u, k = q >> 4, c = q & 15u;
        const uint32_t first = r0 + c * 8u;
        const uint32_t bytes = first < n ? min(8u, n - first) * 2u : 0u;
        cp_async16(tile + tile_off(k, c, 16), x + static_cast<uint64_t>(k) * x_stride + (bytes ? first : 0u), bytes);
    }
    cp_async_commit();
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Copy a row-major fp16 matrix [rows][cols] from global memory into an interleaved tile with
// 16-byte asynchronous copies: every chunk of every weight matrix is in flight at once (a
// load-then-store loop through registers serialises on each load's L2 latency).  The caller
// commits the group and waits for it before the first MMA reads the tile.
__device__ __forceinline__ void load_weight_tile(unsigned char* tile, const __half* W, uint32_t rows, uint32_t cols) {
    const uint32_t cpr = cols / 8u;
    for (uint32_t q = threadIdx.x; q < rows * cpr; q += blockDim.x) {
        const uint32_t r = q / cpr, c = q % cpr;
        cp_async16(tile + tile_off(r, c, cpr), W + r * cols + c * 8u, 16u);
    }
}

// Two fp32 values to packed fp16 (a low, b high), rounded to nearest, negative values to +0: one
// cvt.rn.relu.f16x2.f32 instead of two max + one conversion.
__device__ __forceinline__ uint32_t pack2_relu(float a, float b) {
    uint32_t d;
    asm("cvt.rn.relu.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(b), "f"(a));
    return d;
}

// Store 8*nchunks fp32 values of this thread's row (ReLU optional) as fp16 into a tile.
template <uint32_t NCHUNK, bool RELU>
__device__ __forceinline__ void store_row(unsigned char* tile, uint32_t r, const float* v) {
#pragma unroll
    for (uint32_t c = 0; c < NCHUNK; ++c) {
        const float* a = v + c * 8;
        if constexpr (RELU)
            store_chunk(tile, r, c, NCHUNK, make_uint4(pack2_relu(a[0], a[1]), pack2_relu(a[2], a[3]), pack2_relu(a[4], a[5]), pack2_relu(a[6], a[7])));
        else
            store_chunk(tile, r, c, NCHUNK, make_uint4(pack2(a[0], a[1]), pack2(a[2], a[3]), pack2(a[4], a[5]), pack2(a[6], a[7])));
    }
}

// Store a row of 32 fp16 values (already rounded) into a 4-chunk tile.
__device__ __forceinline__ void store_row_half32(unsigned char* tile, uint32_t r, const unsigned short* x) {
#pragma unroll
    for (uint32_t c = 0; c < 4; ++c) {
        const unsigned short* h = x + c * 8;
        store_chunk(tile, r, c, 4,
                    make_uint4(h[0] | (static_cast<uint32_t>(h[1]) << 16), h[2] | (static_cast<uint32_t>(h[3]) << 16),
                               h[4] | (static_cast<uint32_t>(h[5]) << 16), h[6] | (static_cast<uint32_t>(h[7]) << 16)));
    }
}

// Read N fp32 accumulator columns [col, col+N) of this thread's lane.
// All N / 16 reads are issued before the one wait, so their latencies overlap.
template <uint32_t N>
__device__ __forceinline__ void read_acc(uint32_t tmem, uint32_t col, float* v) {
    const uint32_t lane_base = (threadIdx.x & ~31u) << 16;
    uint32_t r[N / 16][16];
#pragma unroll
    for (uint32_t c = 0; c < N / 16; ++c) umma::tmem_ld16_async(tmem + lane_base + col + c * 16, r[c]);
    umma::tmem_wait_ld();
#pragma unroll
    for (uint32_t c = 0; c < N / 16; ++c)
#pragma unroll
        for (int j = 0; j < 16; ++j) v[c * 16 + j] = __uint_as_float(r[c][j]);
}

// Issue D(+)= A * B^T over K (multiple of 16) from one thread.
// A: M=128 rows.  K-major A: tile rows = M, cpr chunks per row.  MN-major A: tile rows = K.
// B: N rows.       K-major B: tile rows = N.                     MN-major B: tile rows = K.
__device__ __forceinline__ void gemm(uint32_t d_tmem, uint32_t N, uint32_t K, uint32_t a_saddr, bool a_mn, uint32_t a_cpr,
                                     uint32_t b_saddr, bool b_mn, uint32_t b_cpr, bool accumulate) {
    const uint32_t a_lbo = a_mn ? 128u * a_cpr : 128u, a_sbo = a_mn ? 128u : 128u * a_cpr;
    const uint32_t b_lbo = b_mn ? 128u * b_cpr : 128u, b_sbo = b_mn ? 128u : 128u * b_cpr;
    const uint32_t idesc = umma::make_idesc_f16(128u, N, a_mn, b_mn);
    for (uint32_t ks = 0; ks < K / 16u; ++ks) {
        const uint64_t ad = umma::make_desc(a_saddr + ks * 2u * a_lbo, a_lbo, a_sbo);
        const uint64_t bd = umma::make_desc(b_saddr + ks * 2u * b_lbo, b_lbo, b_sbo);
        umma::mma_f16(d_tmem, ad, bd, idesc, (accumulate || ks > 0) ? 1u : 0u);
    }
}

// Issue D(+)= A * B^T over K (multiple of 16) from one thread, A (128 rows x K fp16) read from
// tensor memory at a_tmem (8 columns per K step of 16), B K-major in shared memory.
__device__ __forceinline__ void gemm_ta(uint32_t d_tmem, uint32_t N, uint32_t K, uint32_t a_tmem, uint32_t b_saddr, uint32_t b_cpr) {
    const uint32_t idesc = umma::make_idesc_f16(128u, N, false, false);
    for (uint32_t ks = 0; ks < K / 16u; ++ks) {
        const uint64_t bd = umma::make_desc(b_saddr + ks * 256u, 128u, 128u * b_cpr);
        umma::mma_f16_ta(d_tmem, a_tmem + ks * 8u, bd, idesc, ks > 0 ? 1u : 0u);
    }
}

// Store 8*NCHUNK fp32 values of this thread's row (ReLU optional) as fp16 into its TMEM lane,
// from column col on (two values per column, the even one low): the A operand of the next
// layer's MMA.  NCHUNK is 4 or 8 (16 or 32 columns).  Waits for its own stores.
template <uint32_t NCHUNK, bool RELU>
__device__ __forceinline__ void store_row_tmem(uint32_t tmem, uint32_t col, const float* v) {
    const uint32_t lane_base = (threadIdx.x & ~31u) << 16;
#pragma unroll
    for (uint32_t g = 0; g < NCHUNK / 4; ++g) {
        uint32_t r[16];
#pragma unroll
        for (uint32_t j = 0; j < 16; ++j) r[j] = RELU ? pack2_relu(v[g * 32 + 2 * j], v[g * 32 + 2 * j + 1]) : pack2(v[g * 32 + 2 * j], v[g * 32 + 2 * j + 1]);
        umma::tmem_st16(tmem + lane_base + col + g * 16u, r);
    }
    umma::tmem_wait_st();
}

// Store a row of 32 fp16 values (already rounded) into this thread's TMEM lane at column col.
__device__ __forceinline__ void store_half32_tmem(uint32_t tmem, uint32_t col, const unsigned short* x) {
    uint32_t r[16];
#pragma unroll
    for (uint32_t j = 0; j < 16; ++j) r[j] = x[2 * j] | (static_cast<uint32_t>(x[2 * j + 1]) << 16);
    umma::tmem_st16(tmem + ((threadIdx.x & ~31u) << 16) + col, r);
    umma::tmem_wait_st();
}

// All threads' TMEM stores (or reads) are complete before the MMA issued after it.
__device__ __forceinline__ void stage_sync_tmem() {
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
}

// Degree-4 SH of dir = 2 * warped - 1 (ngp.train.cu:962-993), one IEEE operation at a time with
// explicit fused multiply-adds for the a*b+c forms.
__device__ __forceinline__ void sh16(float wx, float wy, float wz, float (&o)[16]) {
    const float x = __fsub_rn(__fmul_rn(wx, 2.0f), 1.0f), y = __fsub_rn(__fmul_rn(wy, 2.0f), 1.0f), z = __fsub_rn(__fmul_rn(wz, 2.0f), 1.0f);
    const float xy = __fmul_rn(x, y), xz = __fmul_rn(x, z), yz = __fmul_rn(y, z);
    const float x2 = __fmul_rn(x, x), y2 = __fmul_rn(y, y), z2 = __fmul_rn(z, z);
    o[0]  = 0.28209479177387814f;
    o[1]  = __fmul_rn(-0.48860251190291987f, y);
    o[2]  = __fmul_rn(0.48860251190291987f, z);
    o[3]  = __fmul_rn(-0.48860251190291987f, x);
    o[4]  = __fmul_rn(1.0925484305920792f, xy);
    o[5]  = __fmul_rn(-1.0925484305920792f, yz);
    o[6]  = __fmaf_rn(0.94617469575755997f, z2, -0.31539156525251999f);
    o[7]  = __fmul_rn(-1.0925484305920792f, xz);
    o[8]  = __fmaf_rn(0.54627421529603959f, x2, -__fmul_rn(0.54627421529603959f, y2));
    o[9]  = __fmul_rn(__fmul_rn(0.59004358992664352f, y), __fmaf_rn(-3.0f, x2, y2));
    o[10] = __fmul_rn(__fmul_rn(2.8906114426405538f, xy), z);
    o[11] = __fmul_rn(__fmul_rn(0.45704579946446572f, y), __fmaf_rn(-5.0f, z2, 1.0f));
    o[12] = __fmul_rn(__fmul_rn(0.3731763325901154f, z), __fmaf_rn(5.0f, z2, -3.0f));
    o[13] = __fmul_rn(__fmul_rn(0.45704579946446572f, x), __fmaf_rn(-5.0f, z2, 1.0f));
    o[14] = __fmul_rn(__fmul_rn(1.4453057213202769f, z), __fsub_rn(x2, y2));
    o[15] = __fmul_rn(__fmul_rn(0.59004358992664352f, x), __fmaf_rn(3.0f, y2, -x2));
}

// CTA-wide step boundary: make this thread's shared-memory writes visible to the tensor core,
// order its earlier TMEM reads before the barrier, and synchronise.
__device__ __forceinline__ void stage_sync() {
    umma::fence_proxy_async();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
}

// Wait for the MMAs committed to `mbar` (phase parity flips every call).
__device__ __forceinline__ bool stage_wait(uint64_t* mbar, uint32_t& phase) {
    const bool ok = umma::mbar_wait(mbar, phase);
    phase ^= 1u;
    umma::fence_after_sync();
    if (!ok) atomicOr(&g_mlp_status, 1u);
    return ok;
}

// One row's global inputs: 32 fp16 features (feature-major source, coalesced across a warp per
// feature) and, when the colour network runs, the warped view direction of its record.
// A row list (optional) maps tile row r to sample rows[r]: its features, record and output are
// read and written at that sample's position.
template <bool DIR, bool XROWS = false>
struct RowInputs {
    unsigned short x[XROWS ? 1 : 32];  // register-gathered inputs only (none when the tile arrives by cp.async)
    float dir[DIR ? 3 : 1];
    uint32_t col;  // the sample this row reads and writes
};

template <bool DIR, bool XROWS = false>
__device__ __forceinline__ void load_row_inputs(const __half* __restrict__ x, uint32_t x_stride, const float* __restrict__ coords,
                                                uint32_t coord_stride, uint32_t n, uint32_t row, RowInputs<DIR, XROWS>& in,
                                                const uint32_t* __restrict__ rows = nullptr) {
    const bool valid = row < n;
    in.col           = valid ? (rows != nullptr ? __ldg(rows + row) : row) : 0u;
    const unsigned short* xs = reinterpret_cast<const unsigned short*>(x);
    if constexpr (!XROWS) {
#pragma unroll
        for (uint32_t k = 0; k < 32; ++k) in.x[k] = valid ? __ldg(xs + static_cast<uint64_t>(k) * x_stride + in.col) : static_cast<unsigned short>(0);
    }
    if constexpr (DIR) {
        const float* c = coords + static_cast<uint64_t>(in.col) * coord_stride;
        in.dir[0] = __ldg(c + 4), in.dir[1] = __ldg(c + 5), in.dir[2] = __ldg(c + 6);
    }
}

struct MlpForwardParams {
    uint32_t n;
    const __half* params;   // packed MLP weights (10,240 halves)
    const __half* x;        // encoded positions, feature-major [32][x_stride]
    uint32_t x_stride;
    const float* coords;    // sample records (view direction at floats 4..6)
    uint32_t coord_stride;
    __half* out;            // [n][16] row-major (MODE full) or [n] raw density (MODE density)
    __half* density_rgb_in; // optional: density outputs, feature-major [16][x_stride]
    const uint32_t* rows;   // optional row list (see RowInputs)
    const uint32_t* n_dev;  // optional device-side row count (<= n)
    // optional (density mode): the density-grid splat (K3) of row i's density into
    // splat_scratch[splat_indices[i]] instead of writing out
    const uint32_t* splat_indices;
    float* splat_scratch;
};

enum : int { kModeFull = 0, kModeDensity = 1 };
// how a forward kernel reads its inputs: feature-major through registers (any row list),
// row-major by cp.async, or feature-major contiguous rows by cp.async
enum : int { kXRegs = 0, kXRows = 1, kXCols = 2 };

// TMEM columns: D0 (64-wide accumulator) 0-63, D1 (16-wide) 64-79, and the A operand of the
// hidden layers (128 rows x up to 64 fp16 = 32 columns) at kFwdA: activations never pass
// through shared memory.
constexpr uint32_t kFwdTmemCols = 128, kFwdA = 96;
// weights | a ring of up to four 8 KB input tiles (cp.async inputs: the next tiles' copies land there)
constexpr uint32_t kFwdSmem     = kSWeights + 4 * 8192 + 1024;

// The density network alone (two layers) is light: 64 TMEM columns (D0 0-63; its ReLU output
// goes back into columns 32-63 as the A operand of the output layer, whose 16-wide result lands
// in columns 0-15), only its two weight matrices and a small input ring in shared memory, so
// that up to six CTAs share an SM and more tile chains overlap.
constexpr uint32_t kDensTmemCols = 64, kDensA = 32, kDensXBase = kSWdOut + 2048;
__host__ __device__ constexpr uint32_t fwd_ahead(int mode, int xin) { return (xin == kXCols && mode == kModeDensity) ? 2u : 1u; }
__host__ __device__ constexpr uint32_t fwd_smem(int mode, int xin) {
    return mode == kModeDensity ? kDensXBase + (fwd_ahead(mode, xin) + 1u) * 8192u + 1024u : kFwdSmem;
}

// resident CTAs per SM the register allocation must allow
template <int MODE, int XIN>
constexpr int kFwdMinCtas = MODE == kModeDensity ? (XIN == kXRegs ? 5 : 6) : 4;

template <int MODE, int XIN>
__global__ void __launch_bounds__(kThreads, kFwdMinCtas<MODE, XIN>) mlp_forward_kernel(const __grid_constant__ MlpForwardParams p) {
    constexpr bool XROWS  = XIN == kXRows;
    constexpr bool XASYNC = XIN != kXRegs;  // inputs staged by cp.async
    constexpr bool DENS   = MODE == kModeDensity;
    // tiles in flight ahead of the one computed: the density network's two layers take less time
    // than a tile's DRAM reads, so its contiguous inputs are fetched two tiles ahead
    constexpr uint32_t kAhead = fwd_ahead(MODE, XIN);
    constexpr uint32_t kBufs  = kAhead + 1u;
    constexpr uint32_t kCols  = DENS ? kDensTmemCols : kFwdTmemCols;
    constexpr uint32_t kA     = DENS ? kDensA : kFwdA;  // TMEM column of the hidden layers' A operand
    constexpr uint32_t kD1    = DENS ? 0u : 64u;        // TMEM column of the 16-wide output accumulator
    extern __shared__ __align__(1024) unsigned char smem[];
    unsigned char* sw    = smem;                      // weights
    // input tiles: a ring of kBufs tiles of 128 x 32, tile b at sxb(b) (an offset, not an indexed
    // array, so the choice stays in registers); the density network's register-gathered inputs
    // are stored into tile 0
    auto sxb = [&](uint32_t b) { return smem + (DENS ? kDensXBase : kSWeights) + (b % kBufs) * 8192u; };
    __shared__ uint64_t mbar;
    __shared__ uint32_t tmem_slot;

    const uint32_t t = threadIdx.x;
    MLP_TRACE(0);
    load_weight_tile(sw + kSWdIn, p.params + kWdIn, 64, 32);
    load_weight_tile(sw + kSWdOut, p.params + kWdOut, 16, 64);
    if (MODE == kModeFull) {
        load_weight_tile(sw + kSWrIn, p.params + kWrIn, 64, 32);
        load_weight_tile(sw + kSWrH, p.params + kWrH, 64, 64);
        load_weight_tile(sw + kSWrOut, p.params + kWrOut, 16, 64);
    }
    cp_async_commit();  // the weights: waited for with the first tile's inputs
    const uint32_t n       = p.n_dev != nullptr ? min(*p.n_dev, p.n) : p.n;
    const uint32_t n_tiles = (n + kRows - 1) / kRows;

    // The next tile's inputs are loaded into registers while this tile's layers run (software
    // pipelining of the only global-memory reads of the loop).
    // Row-major inputs (kXRows) and feature-major inputs of contiguous rows (kXCols) arrive by
    // cp.async one tile ahead into the other input buffer; feature-major inputs of a row list
    // (kXRegs) are gathered into registers one tile ahead.
    // The first tile's loads are in flight with the weights' during the set-up below.
    RowInputs<MODE == kModeFull, XASYNC> cur, nxt;
    if (blockIdx.x < n_tiles) {
        load_row_inputs(p.x, p.x_stride, p.coords, p.coord_stride, n, blockIdx.x * kRows + t, cur, p.rows);
        if constexpr (XROWS) issue_row_copy(sxb(0), t, p.x, cur.col, blockIdx.x * kRows + t < n);
        if constexpr (XIN == kXCols) issue_col_copy(sxb(0), p.x, p.x_stride, blockIdx.x * kRows, n);
    } else if constexpr (XASYNC) {
        cp_async_commit();
    }
#pragma unroll
    for (uint32_t j = 1; j < kAhead; ++j) {  // deeper rings: tiles 1 .. kAhead - 1 as well
        if (blockIdx.x + j * gridDim.x < n_tiles)
            issue_col_copy(sxb(j), p.x, p.x_stride, (blockIdx.x + j * gridDim.x) * kRows, n);
        else
            cp_async_commit();
    }
    if (t < 32) umma::tmem_alloc(&tmem_slot, kCols);
    if (t == 0) umma::mbar_init(&mbar, 1);
    stage_sync();
    MLP_TRACE(1);
    const uint32_t tmem = tmem_slot;
    const uint32_t d0 = tmem, d1 = tmem + kD1;
    const uint32_t a_act = tmem + kA, a_sw = umma::smem_addr(sw);
    uint32_t phase  = 0;
    bool ok         = true;
    uint32_t it = 0;
    for (uint32_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const uint32_t row   = tile * kRows + t;
        const bool valid     = row < n;
        const uint32_t a_sx  = umma::smem_addr(sxb(XASYNC ? it : 0u));  // input tile in shared memory
        if (tile + gridDim.x < n_tiles) {
            load_row_inputs(p.x, p.x_stride, p.coords, p.coord_stride, n, (tile + gridDim.x) * kRows + t, nxt, p.rows);
            if constexpr (XROWS) issue_row_copy(sxb(it + 1u), t, p.x, nxt.col, (tile + gridDim.x) * kRows + t < n);
        }
        if constexpr (XIN == kXCols) {
            if (tile + kAhead * gridDim.x < n_tiles)
                issue_col_copy(sxb(it + kAhead), p.x, p.x_stride, (tile + kAhead * gridDim.x) * kRows, n);
            else
                cp_async_commit();  // an empty group keeps the wait count below uniform
        } else if constexpr (XROWS) {
            if (tile + gridDim.x >= n_tiles) cp_async_commit();
        }
        // ---- input row: 32 fp16 features ----
        if constexpr (XASYNC)
            cp_async_wait<kAhead>();  // this tile's copies (all but the kAhead groups issued after them) have landed
        else {
            cp_async_wait<0>();  // the weights (first tile only; later tiles have none pending)
            if constexpr (DENS)
                store_row_half32(sxb(0), t, cur.x);  // (its TMEM holds no room beside D0)
            else
                store_half32_tmem(tmem, kFwdA, cur.x);
        }
        MLP_TRACE(2 + it * 8);
        stage_sync();
        if (t == 0) {
            if constexpr (XROWS || (DENS && XIN == kXRegs))
                gemm(d0, 64, 32, a_sx, false, 4, a_sw + kSWdIn, false, 4, false);
            else if constexpr (XIN == kXCols)
                gemm(d0, 64, 32, a_sx, true, 16, a_sw + kSWdIn, false, 4, false);  // MN-major A
            else
                gemm_ta(d0, 64, 32, a_act, a_sw + kSWdIn, 4);
            umma::commit(&mbar);
        }
        ok = stage_wait(&mbar, phase);
        MLP_TRACE(2 + it * 8 + 1);
        {
            float h[64];
            read_acc<64>(tmem, 0, h);
            store_row_tmem<8, true>(tmem, kA, h);
        }
        stage_sync_tmem();
        if (t == 0) {
            gemm_ta(d1, 16, 64, a_act, a_sw + kSWdOut, 8);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        MLP_TRACE(2 + it * 8 + 2);
        float dens[16];
        read_acc<16>(tmem, kD1, dens);
        if (MODE == kModeDensity) {
            if (valid) {
                const __half d = __float2half_rn(dens[0]);
                if (p.splat_scratch != nullptr) {
                    // K3 (ngp.train.cu:426-432) on the rounded density, as splat_kernel computes it
                    const float thickness = expf(__half2float(d)) * kConeStep;
                    atomicMax(reinterpret_cast<uint32_t*>(p.splat_scratch + __ldg(p.splat_indices + cur.col)), __float_as_uint(thickness));
                } else {
                    p.out[cur.col] = d;
                }
            }
            cur = nxt;
            MLP_TRACE(2 + it * 8 + 7);
            umma::fence_before_sync();
            if (!__syncthreads_and(ok)) break;
            umma::fence_after_sync();
            continue;
        }
        // ---- colour network input: [16 density outputs | 16 SH of the view direction] ----
        {
            float ri[32];
            float sh[16];
            sh16(cur.dir[0], cur.dir[1], cur.dir[2], sh);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                ri[k]      = dens[k];
                ri[16 + k] = sh[k];
            }
            store_row_tmem<4, false>(tmem, kFwdA, ri);
            if (p.density_rgb_in != nullptr && valid)
#pragma unroll
                for (int k = 0; k < 16; ++k) p.density_rgb_in[static_cast<uint64_t>(k) * p.x_stride + cur.col] = __float2half_rn(dens[k]);
        }
        stage_sync_tmem();
        if (t == 0) {
            gemm_ta(d0, 64, 32, a_act, a_sw + kSWrIn, 4);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        MLP_TRACE(2 + it * 8 + 3);
        {
            float h[64];
            read_acc<64>(tmem, 0, h);
            store_row_tmem<8, true>(tmem, kFwdA, h);
        }
        stage_sync_tmem();
        if (t == 0) {
            gemm_ta(d0, 64, 64, a_act, a_sw + kSWrH, 8);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        MLP_TRACE(2 + it * 8 + 4);
        {
            float h[64];
            read_acc<64>(tmem, 0, h);
            store_row_tmem<8, true>(tmem, kFwdA, h);  // the layer-2 MMA that read them has completed
        }
        stage_sync_tmem();
        if (t == 0) {
            gemm_ta(d1, 16, 64, a_act, a_sw + kSWrOut, 8);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        MLP_TRACE(2 + it * 8 + 5);
        float o[16];
        read_acc<16>(tmem, 64, o);
        o[3] = dens[0];
        if (valid) {
            uint4* dst = reinterpret_cast<uint4*>(p.out + static_cast<uint64_t>(cur.col) * 16u);
            dst[0]     = make_uint4(pack2(o[0], o[1]), pack2(o[2], o[3]), pack2(o[4], o[5]), pack2(o[6], o[7]));
            dst[1]     = make_uint4(pack2(o[8], o[9]), pack2(o[10], o[11]), pack2(o[12], o[13]), pack2(o[14], o[15]));
        }
        cur = nxt;
        MLP_TRACE(2 + it * 8 + 7);
        // a timed-out wait anywhere in the CTA ends the loop for every thread together
        umma::fence_before_sync();
        if (!__syncthreads_and(ok)) break;
        umma::fence_after_sync();
    }
    cp_async_wait<0>();  // no copy (weights or inputs) may still target shared memory at exit
    umma::fence_before_sync();
    __syncthreads();
    if (t < 32) umma::tmem_dealloc(tmem, kCols);
    MLP_TRACE(63);
}

// ---------------------------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------------------------
struct MlpBackwardParams {
    uint32_t n;
    const __half* params;
    const __half* x;          // encoded positions [32][x_stride]
    uint32_t x_stride;
    const float* coords;
    uint32_t coord_stride;
    const __half* dy;         // dL/d(network output) [n][16]: ch 0-2 rgb, ch 3 density
    __half* dx;               // dL/d(encoded positions) [32][dx_stride] (may be null)
    uint32_t dx_stride;
    float* dw_partial;        // [gridDim.x][10240] per-CTA weight-gradient partials
    const uint32_t* rows;     // optional: batch row r reads features and record of sample rows[r]
};

// TMEM columns: D0 working accumulator 0-63; weight-gradient accumulators after it.
constexpr uint32_t kColD0 = 0, kColWrOut = 64, kColWrH = 80, kColWrIn = 144, kColWdOut = 176, kColWdIn = 192;
constexpr uint32_t kBwdTmemCols = 256;
// shared memory tiles (bytes)
// (kBX2: the second input tile; row-major inputs of the next tile are copied into the tile the
// current one does not use)
constexpr uint32_t kBX = kSWeights, kBHd = kBX + 8192, kBRi = kBHd + 16384, kBH1 = kBRi + 8192, kBH2 = kBH1 + 16384, kBDy = kBH2 + 16384,
                   kBGuard = kBDy + 4096, kBX2 = kBGuard + 4096, kBwdSmem = kBX2 + 8192;

template <bool XROWS>
__global__ void __launch_bounds__(kThreads) mlp_backward_kernel(const __grid_constant__ MlpBackwardParams p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ uint64_t mbar;
    __shared__ uint32_t tmem_slot;
    const uint32_t t = threadIdx.x;

    load_weight_tile(smem + kSWdIn, p.params + kWdIn, 64, 32);
    load_weight_tile(smem + kSWdOut, p.params + kWdOut, 16, 64);
    load_weight_tile(smem + kSWrIn, p.params + kWrIn, 64, 32);
    load_weight_tile(smem + kSWrH, p.params + kWrH, 64, 64);
    load_weight_tile(smem + kSWrOut, p.params + kWrOut, 16, 64);
    cp_async_commit();  // the weights: waited for with the first tile's inputs
    // the padded (M = 128) weight-gradient GEMMs read up to 2 KB past the last activation tile
    for (uint32_t i = t; i < 4096 / 16; i += kThreads) reinterpret_cast<uint4*>(smem + kBGuard)[i] = make_uint4(0, 0, 0, 0);
    const uint32_t n_tiles = (p.n + kRows - 1) / kRows;

    // next tile's inputs (features, direction, output gradient) prefetched during this tile; the
    // first tile's loads are in flight with the weights' during the set-up below
    RowInputs<true, XROWS> cur, nxt;
    uint2 dy_cur = make_uint2(0, 0), dy_nxt = make_uint2(0, 0);
    auto load_dy = [&](uint32_t r) {
        return r < p.n ? __ldg(reinterpret_cast<const uint2*>(p.dy + static_cast<uint64_t>(r) * 16u)) : make_uint2(0, 0);
    };
    auto xbuf = [&](uint32_t b) { return smem + ((b & 1u) ? kBX2 : kBX); };
    if (blockIdx.x < n_tiles) {
        load_row_inputs(p.x, p.x_stride, p.coords, p.coord_stride, p.n, blockIdx.x * kRows + t, cur, p.rows);
        if constexpr (XROWS) issue_row_copy(xbuf(0), t, p.x, cur.col, blockIdx.x * kRows + t < p.n);
        dy_cur = load_dy(blockIdx.x * kRows + t);
    }
    if (t < 32) umma::tmem_alloc(&tmem_slot, kBwdTmemCols);
    if (t == 0) umma::mbar_init(&mbar, 1);
    stage_sync();
    const uint32_t tmem = tmem_slot;
    const uint32_t s0   = umma::smem_addr(smem);
    uint32_t phase      = 0;
    bool ok             = true;
    bool first          = true;
    uint32_t it = 0;
    for (uint32_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++it) {
        const uint32_t row = tile * kRows + t;
        const bool valid   = row < p.n;
        const uint32_t bx  = XROWS && (it & 1u) ? kBX2 : kBX;  // this tile's input tile
        if (tile + gridDim.x < n_tiles) {
            load_row_inputs(p.x, p.x_stride, p.coords, p.coord_stride, p.n, (tile + gridDim.x) * kRows + t, nxt, p.rows);
            if constexpr (XROWS) issue_row_copy(xbuf(it + 1u), t, p.x, nxt.col, (tile + gridDim.x) * kRows + t < p.n);
            dy_nxt = load_dy((tile + gridDim.x) * kRows + t);
        } else if constexpr (XROWS) {
            cp_async_commit();  // an empty group keeps the wait count below uniform
        }
        // ---------------- forward recompute ----------------
        if constexpr (XROWS)
            cp_async_wait<1>();  // this tile's copies have landed
        else {
            cp_async_wait<0>();  // the weights (first tile only; later tiles have none pending)
            store_row_half32(smem + kBX, t, cur.x);
        }
        float g[16];
        {
            // rgb output gradient: channels 0-2 (extract_rgb_gradients, ngp.train.cu:1244-1253)
            const uint2 a = dy_cur;
            const __half2* h = reinterpret_cast<const __half2*>(&a);
            const float2 g01 = __half22float2(h[0]), g23 = __half22float2(h[1]);
#pragma unroll
            for (int k = 0; k < 16; ++k) g[k] = 0.0f;
            g[0] = g01.x;
            g[1] = g01.y;
            g[2] = g23.x;
            g[3] = g23.y;  // density gradient, added to the density-output gradient below
        }
        stage_sync();
        if (t == 0) {
            gemm(tmem + kColD0, 64, 32, s0 + bx, false, 4, s0 + kSWdIn, false, 4, false);
            umma::commit(&mbar);
        }
        ok = stage_wait(&mbar, phase);
        {
            float h[64];
            read_acc<64>(tmem, kColD0, h);
            store_row<8, true>(smem + kBHd, t, h);
        }
        stage_sync();
        if (t == 0) {
            gemm(tmem + kColD0, 16, 64, s0 + kBHd, false, 8, s0 + kSWdOut, false, 8, false);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        {
            float ri[32], dens[16], sh[16];
            read_acc<16>(tmem, kColD0, dens);
            sh16(cur.dir[0], cur.dir[1], cur.dir[2], sh);
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                ri[k]      = dens[k];
                ri[16 + k] = sh[k];
            }
            store_row<4, false>(smem + kBRi, t, ri);
        }
        stage_sync();
        if (t == 0) {
            gemm(tmem + kColD0, 64, 32, s0 + kBRi, false, 4, s0 + kSWrIn, false, 4, false);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        {
            float h[64];
            read_acc<64>(tmem, kColD0, h);
            store_row<8, true>(smem + kBH1, t, h);
        }
        stage_sync();
        if (t == 0) {
            gemm(tmem + kColD0, 64, 64, s0 + kBH1, false, 8, s0 + kSWrH, false, 8, false);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        {
            float h[64];
            read_acc<64>(tmem, kColD0, h);
            store_row<8, true>(smem + kBH2, t, h);
            // rgb output gradient tile (K = 16): channels 0-2, zeros elsewhere
            float gy[16];
#pragma unroll
            for (int k = 0; k < 16; ++k) gy[k] = k < 3 ? g[k] : 0.0f;
            store_row<2, false>(smem + kBDy, t, gy);
        }
        // ---------------- backward ----------------
        // B1: dH2 = dY * Wr_out (N = 64, K = 16);  dWr_out^T[i][o] += sum_m H2[m][i] dY[m][o]
        stage_sync();
        if (t == 0) {
            gemm(tmem + kColD0, 64, 16, s0 + kBDy, false, 2, s0 + kSWrOut, true, 8, false);
            gemm(tmem + kColWrOut, 16, 128, s0 + kBH2, true, 8, s0 + kBDy, true, 2, !first);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        {
            float d[64];
            read_acc<64>(tmem, kColD0, d);
#pragma unroll
            for (uint32_t c = 0; c < 8; ++c) {
                const uint4 hv = load_chunk(smem + kBH2, t, c, 8);
                const __half* hh = reinterpret_cast<const __half*>(&hv);
#pragma unroll
                for (int j = 0; j < 8; ++j) d[c * 8 + j] = __half2float(hh[j]) > 0.0f ? d[c * 8 + j] : 0.0f;
            }
            store_row<8, false>(smem + kBH2, t, d);  // dH2 replaces H2 (both MMAs reading H2 are done)
        }
        // B2: dH1 = dH2 * Wr_h (N = 64, K = 64);  dWr_h[o][i] += sum_m dH2[m][o] H1[m][i]
        stage_sync();
        if (t == 0) {
            gemm(tmem + kColD0, 64, 64, s0 + kBH2, false, 8, s0 + kSWrH, true, 8, false);
            gemm(tmem + kColWrH, 64, 128, s0 + kBH2, true, 8, s0 + kBH1, true, 8, !first);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        {
            float d[64];
            read_acc<64>(tmem, kColD0, d);
#pragma unroll
            for (uint32_t c = 0; c < 8; ++c) {
                const uint4 hv = load_chunk(smem + kBH1, t, c, 8);
                const __half* hh = reinterpret_cast<const __half*>(&hv);
#pragma unroll
                for (int j = 0; j < 8; ++j) d[c * 8 + j] = __half2float(hh[j]) > 0.0f ? d[c * 8 + j] : 0.0f;
            }
            store_row<8, false>(smem + kBH1, t, d);  // dH1 replaces H1
        }
        // B3: dRi = dH1 * Wr_in (N = 32, K = 64);  dWr_in[o][i] += sum_m dH1[m][o] Ri[m][i]
        stage_sync();
        if (t == 0) {
            gemm(tmem + kColD0, 32, 64, s0 + kBH1, false, 8, s0 + kSWrIn, true, 4, false);
            gemm(tmem + kColWrIn, 32, 128, s0 + kBH1, true, 8, s0 + kBRi, true, 4, !first);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        {
            float d[32];
            read_acc<32>(tmem, kColD0, d);
            d[0] += g[3];  // add_density_gradient_kernel (ngp.train.cu:1255-1259)
            store_row<2, false>(smem + kBDy, t, d);  // dDensityOut (16) replaces dY
        }
        // B4: dHd = dDo * Wd_out (N = 64, K = 16);  dWd_out^T[i][o] += sum_m Hd[m][i] dDo[m][o]
        stage_sync();
        if (t == 0) {
            gemm(tmem + kColD0, 64, 16, s0 + kBDy, false, 2, s0 + kSWdOut, true, 8, false);
            gemm(tmem + kColWdOut, 16, 128, s0 + kBHd, true, 8, s0 + kBDy, true, 2, !first);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        {
            float d[64];
            read_acc<64>(tmem, kColD0, d);
#pragma unroll
            for (uint32_t c = 0; c < 8; ++c) {
                const uint4 hv = load_chunk(smem + kBHd, t, c, 8);
                const __half* hh = reinterpret_cast<const __half*>(&hv);
#pragma unroll
                for (int j = 0; j < 8; ++j) d[c * 8 + j] = __half2float(hh[j]) > 0.0f ? d[c * 8 + j] : 0.0f;
            }
            store_row<8, false>(smem + kBHd, t, d);  // dHd replaces Hd
        }
        // B5: dX = dHd * Wd_in (N = 32, K = 64);  dWd_in[o][i] += sum_m dHd[m][o] X[m][i]
        stage_sync();
        if (t == 0) {
            gemm(tmem + kColD0, 32, 64, s0 + kBHd, false, 8, s0 + kSWdIn, true, 4, false);
            gemm(tmem + kColWdIn, 32, 128, s0 + kBHd, true, 8, s0 + bx, true, 4, !first);
            umma::commit(&mbar);
        }
        ok = ok && stage_wait(&mbar, phase);
        {
            float d[32];
            read_acc<32>(tmem, kColD0, d);
            if (valid && p.dx != nullptr)
#pragma unroll
                for (uint32_t k = 0; k < 32; ++k) p.dx[static_cast<uint64_t>(k) * p.dx_stride + row] = __float2half_rn(d[k]);
        }
        first  = false;
        cur    = nxt;
        dy_cur = dy_nxt;
        umma::fence_before_sync();
        if (!__syncthreads_and(ok)) break;
        umma::fence_after_sync();
    }

    cp_async_wait<0>();  // no copy (weights or inputs) may still target shared memory
    // ---- write this CTA's weight-gradient partial (rows 0-63 of the M = 128 accumulators) ----
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    float* part = p.dw_partial + static_cast<uint64_t>(blockIdx.x) * kMlpParams;
    if (t < 64) {
        if (first) {
            // this CTA processed no tile: its partial is zero
            for (uint32_t i = 0; i < 64; ++i) {
                if (i < 32) part[kWdIn + t * 32 + i] = 0.0f, part[kWrIn + t * 32 + i] = 0.0f;
                part[kWrH + t * 64 + i] = 0.0f;
                if (i < 16) part[kWrOut + i * 64 + t] = 0.0f, part[kWdOut + i * 64 + t] = 0.0f;
            }
        } else {
            float v[64];
            read_acc<16>(tmem, kColWrOut, v);  // lane t = hidden unit i, column o: dWr_out[o][i]
            for (uint32_t o = 0; o < 16; ++o) part[kWrOut + o * 64 + t] = v[o];
            read_acc<64>(tmem, kColWrH, v);  // lane t = output unit o: dWr_h[o][i]
            for (uint32_t i = 0; i < 64; ++i) part[kWrH + t * 64 + i] = v[i];
            read_acc<32>(tmem, kColWrIn, v);
            for (uint32_t i = 0; i < 32; ++i) part[kWrIn + t * 32 + i] = v[i];
            read_acc<16>(tmem, kColWdOut, v);
            for (uint32_t o = 0; o < 16; ++o) part[kWdOut + o * 64 + t] = v[o];
            read_acc<32>(tmem, kColWdIn, v);
            for (uint32_t i = 0; i < 32; ++i) part[kWdIn + t * 32 + i] = v[i];
        }
    }
    umma::fence_before_sync();
    __syncthreads();
    if (t < 32) umma::tmem_dealloc(tmem, kBwdTmemCols);
}

// dW[j] = scale * sum over CTAs of partial[cta][j] in a fixed order (deterministic): the CTAs are
// split into kReduceGroups interleaved groups (group g: CTAs g, g + G, ...) summed in CTA order by
// their own threads, then the group sums are added in group order.
constexpr uint32_t kReduceGroups = 8;

__global__ void __launch_bounds__(32 * kReduceGroups) mlp_reduce_partials_kernel(const float* __restrict__ partial, uint32_t n_parts, float scale,
                                                                              float* __restrict__ dw_f32, __half* __restrict__ dw_f16) {
    __shared__ float s_sum[kReduceGroups][32];
    const uint32_t lane = threadIdx.x & 31u, g = threadIdx.x >> 5;
    const uint32_t j    = blockIdx.x * 32u + lane;
    float acc           = 0.0f;
    if (j < kMlpParams)
        for (uint32_t c = g; c < n_parts; c += kReduceGroups) acc += partial[static_cast<uint64_t>(c) * kMlpParams + j];
    s_sum[g][lane] = acc;
    __syncthreads();
    if (g != 0 || j >= kMlpParams) return;
    float total = 0.0f;
#pragma unroll
    for (uint32_t q = 0; q < kReduceGroups; ++q) total += s_sum[q][lane];
    total *= scale;
    if (dw_f32 != nullptr) dw_f32[j] = total;
    if (dw_f16 != nullptr) dw_f16[j] = __float2half_rn(total);
}

__global__ void sh_encode_kernel(uint32_t n, const float* __restrict__ coords, uint32_t coord_stride, __half* __restrict__ out,
                                 uint32_t out_stride) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* c = coords + static_cast<uint64_t>(i) * coord_stride;
    float sh[16];
    sh16(c[4], c[5], c[6], sh);
#pragma unroll
    for (uint32_t k = 0; k < 16; ++k) out[static_cast<uint64_t>(k) * out_stride + i] = __float2half_rn(sh[k]);
}

int mlp_grid(int smem_bytes, const void* kernel, uint32_t n_tiles, uint32_t tmem_cols) {
    // CTAs per SM from shared memory (1 KB per CTA is reserved by the hardware), registers and
    // TMEM columns (512 per SM).
    static int smem_per_sm = [] {
        int device = 0, v = 0;
        cudaGetDevice(&device);
        cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device);
        return v > 0 ? v : 233472;
    }();
    cudaFuncAttributes attr{};
    cudaFuncGetAttributes(&attr, kernel);
    const int per_cta_smem = smem_bytes + static_cast<int>(attr.sharedSizeBytes) + 1024;
    int per_sm            = smem_per_sm / per_cta_smem;
    const int regs        = attr.numRegs > 0 ? attr.numRegs : 64;
    const int by_regs     = 65536 / (regs * static_cast<int>(kThreads));
    per_sm                = per_sm < by_regs ? per_sm : by_regs;
    if (per_sm < 1) per_sm = 1;
    const int by_tmem = static_cast<int>(512u / tmem_cols);
    per_sm            = per_sm < by_tmem ? per_sm : by_tmem;
    // $NGP_MLP_CTAS_PER_SM caps the resident CTAs per SM (measurement of how the kernels scale
    // with the number of tiles in flight)
    static int cap = [] {
        const char* v = std::getenv("NGP_MLP_CTAS_PER_SM");
        return v != nullptr ? std::atoi(v) : 0;
    }();
    if (cap > 0 && per_sm > cap) per_sm = cap;
    const uint32_t g  = static_cast<uint32_t>(per_sm * sm_count());
    return static_cast<int>(n_tiles < g ? n_tiles : g);
}

}  // namespace

uint32_t mlp_backward_max_ctas() {
    // upper bound of the backward grid: TMEM allows 512 / 256 = 2 CTAs per SM
    return static_cast<uint32_t>((512u / kBwdTmemCols) * static_cast<uint32_t>(sm_count()));
}

}  // namespace ngp

using namespace ngp;

namespace {
int ensure_attrs() {
    static int status = [] {
        cudaError_t e = cudaSuccess;
        for (const void* f : {reinterpret_cast<const void*>(mlp_forward_kernel<kModeFull, kXRegs>), reinterpret_cast<const void*>(mlp_forward_kernel<kModeDensity, kXRegs>),
                              reinterpret_cast<const void*>(mlp_forward_kernel<kModeFull, kXRows>), reinterpret_cast<const void*>(mlp_forward_kernel<kModeDensity, kXRows>),
                              reinterpret_cast<const void*>(mlp_forward_kernel<kModeFull, kXCols>), reinterpret_cast<const void*>(mlp_forward_kernel<kModeDensity, kXCols>)})
            if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kFwdSmem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(mlp_backward_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem);
        if (e == cudaSuccess) e = cudaFuncSetAttribute(mlp_backward_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kBwdSmem);
        return static_cast<int>(e);
    }();
    if (status != 0) return fail(NGP_ERR_CUDA, std::string("mlp: cudaFuncSetAttribute: ") + cudaGetErrorString(static_cast<cudaError_t>(status)));
    return NGP_OK;
}
}  // namespace

namespace {
template <int MODE>
int launch_forward(const MlpForwardParams& p, uint32_t n_rows, cudaStream_t stream, const char* what) {
    const uint32_t n_tiles = (n_rows + kRows - 1) / kRows;
    // feature-major inputs of contiguous rows go by cp.async when every 16-byte chunk is aligned
    const bool cols = !rows_layout(p.x_stride) && p.rows == nullptr && (reinterpret_cast<uintptr_t>(p.x) & 15u) == 0u && p.x_stride % 8u == 0u;
    constexpr uint32_t cols_tmem = MODE == kModeDensity ? kDensTmemCols : kFwdTmemCols;
    auto run = [&](auto kernel, uint32_t smem) {
        const int grid = mlp_grid(static_cast<int>(smem), reinterpret_cast<const void*>(kernel), n_tiles, cols_tmem);
        kernel<<<grid, kThreads, smem, stream>>>(p);
    };
    if (rows_layout(p.x_stride))
        run(mlp_forward_kernel<MODE, kXRows>, fwd_smem(MODE, kXRows));
    else if (cols)
        run(mlp_forward_kernel<MODE, kXCols>, fwd_smem(MODE, kXCols));
    else
        run(mlp_forward_kernel<MODE, kXRegs>, fwd_smem(MODE, kXRegs));
    return check_launch(what);
}
}  // namespace

extern "C" int ngp_mlp_forward(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const float* coords,
                               uint32_t coord_stride, uint16_t* out, uint16_t* density_rgb_in, void* stream) {
    clear_error();
    if (n == 0) return NGP_OK;
    if (params == nullptr || x == nullptr || coords == nullptr || out == nullptr) return fail(NGP_ERR_INVALID, "mlp forward: null pointer");
    if ((!rows_layout(x_stride) && x_stride < n) || coord_stride < 7) return fail(NGP_ERR_INVALID, "mlp forward: bad stride");
    NGP_TRY(ensure_attrs());
    MlpForwardParams p{n, reinterpret_cast<const __half*>(params), reinterpret_cast<const __half*>(x), x_stride, coords, coord_stride,
                       reinterpret_cast<__half*>(out), reinterpret_cast<__half*>(density_rgb_in), nullptr, nullptr};
    return launch_forward<kModeFull>(p, n, as_stream(stream), "mlp_forward_kernel");
}

extern "C" int ngp_density_forward(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, uint16_t* out, void* stream) {
    clear_error();
    if (n == 0) return NGP_OK;
    if (params == nullptr || x == nullptr || out == nullptr) return fail(NGP_ERR_INVALID, "density forward: null pointer");
    if (!rows_layout(x_stride) && x_stride < n) return fail(NGP_ERR_INVALID, "density forward: bad stride");
    NGP_TRY(ensure_attrs());
    MlpForwardParams p{n, reinterpret_cast<const __half*>(params), reinterpret_cast<const __half*>(x), x_stride, nullptr, 7,
                       reinterpret_cast<__half*>(out), nullptr, nullptr, nullptr};
    return launch_forward<kModeDensity>(p, n, as_stream(stream), "mlp_forward_kernel<density>");
}

extern "C" int ngp_density_forward_splat(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const uint32_t* indices,
                                         float* scratch, void* stream) {
    clear_error();
    if (n == 0) return NGP_OK;
    if (params == nullptr || x == nullptr || indices == nullptr || scratch == nullptr) return fail(NGP_ERR_INVALID, "density forward splat: null pointer");
    if (!rows_layout(x_stride) && x_stride < n) return fail(NGP_ERR_INVALID, "density forward splat: bad stride");
    NGP_TRY(ensure_attrs());
    MlpForwardParams p{n, reinterpret_cast<const __half*>(params), reinterpret_cast<const __half*>(x), x_stride, nullptr, 7, nullptr, nullptr, nullptr,
                       nullptr, indices, scratch};
    return launch_forward<kModeDensity>(p, n, as_stream(stream), "mlp_forward_kernel<density, splat>");
}

extern "C" int ngp_mlp_forward_rows(uint32_t max_rows, const uint32_t* rows, const uint32_t* n_rows, const uint16_t* params, const uint16_t* x,
                                    uint32_t x_stride, const float* coords, uint32_t coord_stride, uint16_t* out, void* stream) {
    clear_error();
    if (max_rows == 0) return NGP_OK;
    if (rows == nullptr || params == nullptr || x == nullptr || coords == nullptr || out == nullptr)
        return fail(NGP_ERR_INVALID, "mlp forward rows: null pointer");
    if (coord_stride < 7) return fail(NGP_ERR_INVALID, "mlp forward rows: bad stride");
    NGP_TRY(ensure_attrs());
    MlpForwardParams p{max_rows, reinterpret_cast<const __half*>(params), reinterpret_cast<const __half*>(x), x_stride, coords, coord_stride,
                       reinterpret_cast<__half*>(out), nullptr, rows, n_rows};
    return launch_forward<kModeFull>(p, max_rows, as_stream(stream), "mlp_forward_kernel");
}

extern "C" int ngp_density_forward_rows(uint32_t max_rows, const uint32_t* rows, const uint32_t* n_rows, const uint16_t* params, const uint16_t* x,
                                        uint32_t x_stride, uint16_t* out, void* stream) {
    clear_error();
    if (max_rows == 0) return NGP_OK;
    if (rows == nullptr || params == nullptr || x == nullptr || out == nullptr) return fail(NGP_ERR_INVALID, "density forward rows: null pointer");
    NGP_TRY(ensure_attrs());
    MlpForwardParams p{max_rows, reinterpret_cast<const __half*>(params), reinterpret_cast<const __half*>(x), x_stride, nullptr, 7,
                       reinterpret_cast<__half*>(out), nullptr, rows, n_rows};
    return launch_forward<kModeDensity>(p, max_rows, as_stream(stream), "mlp_forward_kernel<density>");
}

extern "C" uint32_t ngp_mlp_backward_scratch_floats(void) { return mlp_backward_max_ctas() * kMlpParams; }

namespace ngp {
namespace {
int mlp_backward_launch(uint32_t n, const uint32_t* rows, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const float* coords,
                        uint32_t coord_stride, const uint16_t* dy, uint16_t* dx, uint32_t dx_stride, float* scratch, size_t scratch_floats,
                        float* dw_f32, uint16_t* dw_f16, float dw_scale, void* stream) {
    if (params == nullptr || x == nullptr || coords == nullptr || dy == nullptr || scratch == nullptr)
        return fail(NGP_ERR_INVALID, "mlp backward: null pointer");
    if ((rows == nullptr && !rows_layout(x_stride) && x_stride < n) || coord_stride < 7 || (dx != nullptr && dx_stride < n))
        return fail(NGP_ERR_INVALID, "mlp backward: bad stride");
    NGP_TRY(ensure_attrs());
    const uint32_t n_tiles = (n + kRows - 1) / kRows;
    const bool xrows       = rows_layout(x_stride);
    const void* kern       = xrows ? reinterpret_cast<const void*>(mlp_backward_kernel<true>) : reinterpret_cast<const void*>(mlp_backward_kernel<false>);
    uint32_t grid          = static_cast<uint32_t>(mlp_grid(kBwdSmem, kern, n_tiles == 0 ? 1 : n_tiles, kBwdTmemCols));
    if (static_cast<size_t>(grid) * kMlpParams > scratch_floats) {
        grid = static_cast<uint32_t>(scratch_floats / kMlpParams);
        if (grid == 0) return fail(NGP_ERR_INVALID, "mlp backward: scratch too small (need ngp_mlp_backward_scratch_floats())");
    }
    MlpBackwardParams p{n, reinterpret_cast<const __half*>(params), reinterpret_cast<const __half*>(x), x_stride, coords, coord_stride,
                        reinterpret_cast<const __half*>(dy), reinterpret_cast<__half*>(dx), dx_stride, scratch, rows};
    if (xrows)
        mlp_backward_kernel<true><<<grid, kThreads, kBwdSmem, as_stream(stream)>>>(p);
    else
        mlp_backward_kernel<false><<<grid, kThreads, kBwdSmem, as_stream(stream)>>>(p);
    NGP_TRY(check_launch("mlp_backward_kernel"));
    mlp_reduce_partials_kernel<<<(kMlpParams + 31) / 32, 32 * kReduceGroups, 0, as_stream(stream)>>>(scratch, grid, dw_scale, dw_f32,
                                                                                                       reinterpret_cast<__half*>(dw_f16));
    return check_launch("mlp_reduce_partials_kernel");
}
}  // namespace
}  // namespace ngp

extern "C" int ngp_mlp_backward(uint32_t n, const uint16_t* params, const uint16_t* x, uint32_t x_stride, const float* coords,
                                uint32_t coord_stride, const uint16_t* dy, uint16_t* dx, uint32_t dx_stride, float* scratch,
                                size_t scratch_floats, float* dw_f32, uint16_t* dw_f16, float dw_scale, void* stream) {
    clear_error();
    return mlp_backward_launch(n, nullptr, params, x, x_stride, coords, coord_stride, dy, dx, dx_stride, scratch, scratch_floats, dw_f32, dw_f16,
                               dw_scale, stream);
}

extern "C" int ngp_mlp_backward_rows(uint32_t n, const uint32_t* rows, const uint16_t* params, const uint16_t* x, uint32_t x_stride,
                                     const float* coords, uint32_t coord_stride, const uint16_t* dy, uint16_t* dx, uint32_t dx_stride,
                                     float* scratch, size_t scratch_floats, float* dw_f32, uint16_t* dw_f16, float dw_scale, void* stream) {
    clear_error();
    if (rows == nullptr) return fail(NGP_ERR_INVALID, "mlp backward rows: null row list");
    return mlp_backward_launch(n, rows, params, x, x_stride, coords, coord_stride, dy, dx, dx_stride, scratch, scratch_floats, dw_f32, dw_f16,
                               dw_scale, stream);
}

extern "C" int ngp_mlp_status(uint32_t* out_status, int reset) {
    clear_error();
    uint32_t v = 0;
    NGP_TRY(check_cuda(cudaMemcpyFromSymbol(&v, g_mlp_status, sizeof(v)), "mlp status read"));
    if (reset) {
        const uint32_t zero = 0;
        NGP_TRY(check_cuda(cudaMemcpyToSymbol(g_mlp_status, &zero, sizeof(zero)), "mlp status reset"));
    }
    if (out_status != nullptr) *out_status = v;
    return NGP_OK;
}

extern "C" int ngp_sh_encode(uint32_t n, const float* coords, uint32_t coord_stride, uint16_t* out, uint32_t out_stride, void* stream) {
    clear_error();
    if (n == 0) return NGP_OK;
    if (coords == nullptr || out == nullptr) return fail(NGP_ERR_INVALID, "sh encode: null pointer");
    if (coord_stride < 7 || out_stride < n) return fail(NGP_ERR_INVALID, "sh encode: bad stride");
    sh_encode_kernel<<<(n + 255) / 256, 256, 0, as_stream(stream)>>>(n, coords, coord_stride, reinterpret_cast<__half*>(out), out_stride);
    return check_launch("sh_encode_kernel");
}
