// Library runtime: per-thread error state, device queries and the hash-grid layout.
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>

#include "common.cuh"

namespace ngp {

namespace {
thread_local std::string g_last_error;
}

std::atomic<uint64_t> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
void set_error(const std::string& message) { g_last_error = message; }
void clear_error() { g_last_error.clear(); }

// Fault injection: countdown[site] > 0 arms the site; the event that brings it to zero fails.
namespace {
std::atomic<int64_t> g_fault_countdown[4] = {};

// $NGP_FAULT_INJECT = "<site>:<n>" (site alloc | launch | collective) arms one site at load.
struct FaultEnv {
    FaultEnv() {
        const char* v = std::getenv("NGP_FAULT_INJECT");
        if (v == nullptr) return;
        const char* colon = std::strchr(v, ':');
        if (colon == nullptr) return;
        const std::string site(v, colon);
        const long long n = std::atoll(colon + 1);
        const int idx     = site == "alloc" ? kFaultAlloc : site == "launch" ? kFaultLaunch : site == "collective" ? kFaultCollective : 0;
        if (idx != 0 && n > 0) g_fault_countdown[idx].store(n);
    }
} g_fault_env;
}  // namespace

bool fault_due(FaultSite site) {
    std::atomic<int64_t>& c = g_fault_countdown[site];
    if (c.load(std::memory_order_relaxed) <= 0) return false;
    return c.fetch_sub(1) == 1;
}

int sm_count() {
    static int cached = [] {
        int device = 0, count = 0;
        if (cudaGetDevice(&device) != cudaSuccess) return 148;
        if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || count <= 0) return 148;
        return count;
    }();
    return cached;
}

}  // namespace ngp

using namespace ngp;

extern "C" const char* ngp_last_error(void) { return g_last_error.c_str(); }

extern "C" uint64_t ngp_kernel_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int ngp_fault_inject(int site, int64_t countdown) {
    clear_error();
    if (site < kFaultAlloc || site > kFaultCollective || countdown < 0) return fail(NGP_ERR_INVALID, "fault inject: bad site or countdown");
    g_fault_countdown[site].store(countdown);
    return NGP_OK;
}

extern "C" const char* ngp_version(void) { return "ngp_b200 0.1 (sm_100a)"; }

// Layout of the hash-grid parameters.  Entry counts follow the reference's
// make_network_parameter_layout (ngp.train.h:44-56): min(res^3, 2^32/2) rounded up to a multiple
// of 8, capped at the hashmap size; the per-level scale generalises the reference's
// `res = base << l, scale = res - 1` (ngp.train.cu:885-886) to a real growth factor as in
// example.py:400-401.
extern "C" int ngp_grid_layout_make(uint32_t n_levels, uint32_t features_per_level, uint32_t log2_hashmap_size, uint32_t base_resolution,
                                    double log2_per_level_scale, ngp_grid_layout* out) {
    clear_error();
    if (out == nullptr) return fail(NGP_ERR_INVALID, "grid layout: out is null");
    if (n_levels == 0 || n_levels > NGP_MAX_LEVELS) return fail(NGP_ERR_INVALID, "grid layout: n_levels must be in [1, 32]");
    if (features_per_level != 1 && features_per_level != 2 && features_per_level != 4 && features_per_level != 8)
        return fail(NGP_ERR_INVALID, "grid layout: features_per_level must be 1, 2, 4 or 8");
    if (log2_hashmap_size < 3 || log2_hashmap_size > 27) return fail(NGP_ERR_INVALID, "grid layout: log2_hashmap_size must be in [3, 27]");
    if (base_resolution < 2 || !std::isfinite(log2_per_level_scale) || log2_per_level_scale < 0.0)
        return fail(NGP_ERR_INVALID, "grid layout: bad base resolution or scale");

    ngp_grid_layout layout{};
    layout.n_levels             = n_levels;
    layout.features_per_level   = features_per_level;
    layout.log2_hashmap_size    = log2_hashmap_size;
    layout.base_resolution      = base_resolution;
    layout.log2_per_level_scale = log2_per_level_scale;

    const uint64_t hashmap_size  = uint64_t{1} << log2_hashmap_size;
    const uint64_t max_positions = std::numeric_limits<uint32_t>::max() / 2ull;
    uint64_t cursor              = 0;
    for (uint32_t l = 0; l < n_levels; ++l) {
        const double scale = std::exp2(static_cast<double>(l) * log2_per_level_scale) * static_cast<double>(base_resolution) - 1.0;
        if (!(scale > 0.0) || scale > 1.0e7) return fail(NGP_ERR_INVALID, "grid layout: level scale out of range");
        const uint64_t res = static_cast<uint64_t>(std::ceil(scale)) + 1u;
        uint64_t dense     = res * res * res;
        if (dense > max_positions) dense = max_positions;
        uint64_t positions = (dense + 7u) / 8u * 8u;
        if (positions > hashmap_size) positions = hashmap_size;
        layout.offsets[l]    = static_cast<uint32_t>(cursor);
        layout.resolution[l] = static_cast<uint32_t>(res);
        layout.scale[l]      = static_cast<float>(scale);
        cursor += positions;
        if (cursor * features_per_level > 0xFFFFFFFFull) return fail(NGP_ERR_INVALID, "grid layout: too many parameters");
    }
    layout.offsets[n_levels] = static_cast<uint32_t>(cursor);
    layout.n_entries         = static_cast<uint32_t>(cursor);
    layout.n_params          = static_cast<uint32_t>(cursor * features_per_level);
    *out                     = layout;
    return NGP_OK;
}
