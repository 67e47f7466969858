// Test driver for include/ngp_b200_dataset.hpp (built by tests/test_cpp_dataset.py, loaded with
// ctypes; no GPU): load a scene with the C++ loaders and copy one split out, or decode one PNG.
// Entry points return 0, or 1 with the message in `err`.
#include <cstdio>
#include <cstring>

#include "ngp_b200_dataset.hpp"

namespace {
int fail(char* err, std::size_t n, const std::string& msg) {
    std::snprintf(err, n, "%s", msg.c_str());
    return 1;
}
}  // namespace

extern "C" {

// kind 0: NeRF-synthetic, 1: DD-NeRF.  counts[3] = frames per split (train, validation, test);
// dims[6] = width, height of each split's first frame.
int probe_dataset_shape(const char* path, int kind, float scale, std::uint32_t* counts, std::uint32_t* dims, char* err, std::size_t en) {
    const auto ds = kind == 0 ? ngp::b200::dataset::load_nerf_synthetic(path, scale) : ngp::b200::dataset::load_dd_nerf_dataset(path, scale);
    if (!ds) return fail(err, en, ds.error());
    const std::vector<ngp::b200::dataset::NGPDataset::Frame>* splits[3] = {&ds->train, &ds->validation, &ds->test};
    for (int s = 0; s < 3; ++s) {
        counts[s]       = static_cast<std::uint32_t>(splits[s]->size());
        dims[2 * s]     = splits[s]->empty() ? 0u : splits[s]->front().width;
        dims[2 * s + 1] = splits[s]->empty() ? 0u : splits[s]->front().height;
    }
    return 0;
}

// One split's frames: pixels [frames][h][w][4], cameras [frames][12], intrinsics [frames][4].
int probe_dataset_split(const char* path, int kind, float scale, int split, std::uint8_t* pixels, float* cameras, float* intrinsics, char* err,
                        std::size_t en) {
    const auto ds = kind == 0 ? ngp::b200::dataset::load_nerf_synthetic(path, scale) : ngp::b200::dataset::load_dd_nerf_dataset(path, scale);
    if (!ds) return fail(err, en, ds.error());
    const auto& frames = split == 0 ? ds->train : split == 1 ? ds->validation : ds->test;
    std::size_t off    = 0;
    for (std::size_t i = 0; i < frames.size(); ++i) {
        std::memcpy(pixels + off, frames[i].rgba.data(), frames[i].rgba.size());
        off += frames[i].rgba.size();
        std::memcpy(cameras + 12 * i, frames[i].camera.data(), 12 * sizeof(float));
        intrinsics[4 * i] = frames[i].focal_x, intrinsics[4 * i + 1] = frames[i].focal_y;
        intrinsics[4 * i + 2] = frames[i].principal_x, intrinsics[4 * i + 3] = frames[i].principal_y;
    }
    return 0;
}

int probe_png(const char* path, std::uint8_t* rgba, std::size_t capacity, std::uint32_t* wh, char* err, std::size_t en) {
    try {
        const auto v = ngp::b200::dataset::detail::load_png_rgba(path, wh[0], wh[1]);
        if (v.size() > capacity) return fail(err, en, "buffer too small");
        std::memcpy(rgba, v.data(), v.size());
        return 0;
    } catch (const std::exception& e) {
        return fail(err, en, e.what());
    }
}

}  // extern "C"
