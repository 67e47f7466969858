// Test driver for include/ngp_b200_train.hpp (built by tests/test_cpp_api.py, loaded with ctypes):
// the host file formats without a GPU, and one InstantNGP lifecycle through the C++23 interface
// on a GPU.  Every entry point returns 0, or 1 with the message in `err`.
#include <cstdio>
#include <cstring>

#include "ngp_b200_train.hpp"

namespace fmt = ngp::b200::train::format;

namespace {

int fail(char* err, std::size_t n, const std::string& msg) {
    std::snprintf(err, n, "%s", msg.c_str());
    return 1;
}

ngp_grid_layout layout_of(std::uint32_t L, std::uint32_t F, std::uint32_t log2T, std::uint32_t base, double log2_scale) {
    ngp_grid_layout g{};
    if (ngp_grid_layout_make(L, F, log2T, base, log2_scale, &g) != NGP_OK) throw std::runtime_error{ngp_last_error()};
    return g;
}

std::vector<ngp::b200::dataset::NGPDataset::Frame> frames(std::uint32_t count, std::uint32_t w, std::uint32_t h, const std::uint8_t* pixels,
                                                          const float* cameras, const float* intrinsics) {
    std::vector<ngp::b200::dataset::NGPDataset::Frame> out(count);
    const std::size_t px = static_cast<std::size_t>(w) * h * 4u;
    for (std::uint32_t i = 0; i < count; ++i) {
        out[i].rgba.assign(pixels + i * px, pixels + (i + 1) * px);
        std::memcpy(out[i].camera.data(), cameras + i * 12u, 12u * sizeof(float));
        out[i].width = w, out[i].height = h;
        out[i].focal_x = intrinsics[0], out[i].focal_y = intrinsics[1], out[i].principal_x = intrinsics[2], out[i].principal_y = intrinsics[3];
    }
    return out;
}

}  // namespace

extern "C" {

int probe_header(std::uint32_t L, std::uint32_t F, std::uint32_t log2T, std::uint32_t base, double log2_scale, float scene_scale, char* out,
                 std::size_t n, char* err, std::size_t en) {
    try {
        const std::string h = fmt::weights_header(layout_of(L, F, log2T, base, log2_scale), scene_scale);
        if (h.size() + 1 > n) return fail(err, en, "buffer too small");
        std::memcpy(out, h.c_str(), h.size() + 1);
        return 0;
    } catch (const std::exception& e) {
        return fail(err, en, e.what());
    }
}

int probe_write_weights(const char* path, const float* params, std::uint32_t L, std::uint32_t F, std::uint32_t log2T, std::uint32_t base,
                        double log2_scale, float scene_scale, char* err, std::size_t en) {
    try {
        fmt::write_weights(path, params, layout_of(L, F, log2T, base, log2_scale), scene_scale);
        return 0;
    } catch (const std::exception& e) {
        return fail(err, en, e.what());
    }
}

int probe_read_weights(const char* path, float* params, std::size_t count, std::uint32_t L, std::uint32_t F, std::uint32_t log2T, std::uint32_t base,
                       double log2_scale, float scene_scale, char* err, std::size_t en) {
    try {
        const std::vector<float> v = fmt::read_weights(path, layout_of(L, F, log2T, base, log2_scale), scene_scale);
        if (v.size() != count) return fail(err, en, "parameter count mismatch");
        std::memcpy(params, v.data(), count * sizeof(float));
        return 0;
    } catch (const std::exception& e) {
        return fail(err, en, e.what());
    }
}

int probe_canonical(const char* json, char* out, std::size_t n, char* err, std::size_t en) {
    try {
        const std::string c = fmt::JsonCanon{json}.canonical();
        if (c.size() + 1 > n) return fail(err, en, "buffer too small");
        std::memcpy(out, c.c_str(), c.size() + 1);
        return 0;
    } catch (const std::exception& e) {
        return fail(err, en, e.what());
    }
}

int probe_write_png(const char* path, const std::uint8_t* rgb, std::uint32_t w, std::uint32_t h, char* err, std::size_t en) {
    try {
        fmt::write_png(path, rgb, w, h);
        return 0;
    } catch (const std::exception& e) {
        return fail(err, en, e.what());
    }
}

// One lifecycle on a GPU: construct, train, validate, test (PNGs into out_dir), export, and a
// second model loading the export.  results: train loss, validation PSNR, test PSNR, test image
// count, params equal after the round trip (1/0), step.
int probe_lifecycle(std::uint32_t w, std::uint32_t h, std::uint32_t n_train, const std::uint8_t* train_px, const float* train_cam,
                    std::uint32_t n_test, const std::uint8_t* test_px, const float* test_cam, const float* intrinsics, std::int32_t steps,
                    const char* out_dir, double* results, char* err, std::size_t en) {
    using ngp::train::InstantNGP;  // the reference's names (aliases of ngp::b200::*)
    try {
        ngp::dataset::NGPDataset ds;
        ds.train       = frames(n_train, w, h, train_px, train_cam, intrinsics);
        ds.validation  = frames(n_test, w, h, test_px, test_cam, intrinsics);
        ds.test        = frames(n_test, w, h, test_px, test_cam, intrinsics);
        ds.scene_scale = ngp::b200::dataset::DEFAULT_SCENE_SCALE;
        InstantNGP model{ds};
        const auto t = model.train(steps);
        if (!t) return fail(err, en, "train: " + t.error());
        const auto v = model.validate();
        if (!v) return fail(err, en, "validate: " + v.error());
        const std::filesystem::path dir{out_dir};
        const auto s = model.test(dir / "test");
        if (!s) return fail(err, en, "test: " + s.error());
        const auto e = model.export_weights(dir / "model.safetensors");
        if (!e) return fail(err, en, "export: " + e.error());
        if (model.load_weights(dir / "model.safetensors")) return fail(err, en, "load after training must fail");
        InstantNGP second{ds};
        const auto l = second.load_weights(dir / "model.safetensors");
        if (!l) return fail(err, en, "load: " + l.error());
        std::vector<float> a(ngp_trainer_param_count(model.handle())), b(a.size());
        ngp_trainer_get_params(model.handle(), a.data(), static_cast<std::uint32_t>(a.size()));
        ngp_trainer_get_params(second.handle(), b.data(), static_cast<std::uint32_t>(b.size()));
        results[0] = t->loss, results[1] = v->psnr, results[2] = s->psnr, results[3] = s->comparison_image_count;
        results[4] = std::memcmp(a.data(), b.data(), a.size() * sizeof(float)) == 0 ? 1.0 : 0.0, results[5] = t->step;
        return 0;
    } catch (const std::exception& e) {
        return fail(err, en, e.what());
    }
}

// Construction errors surface as std::runtime_error with the library's message (the reference's
// constructor throws on a failed device set-up): an empty dataset, or no usable device.
int probe_construct_error(int empty_dataset, char* err, std::size_t en) {
    ngp::b200::dataset::NGPDataset ds;
    if (!empty_dataset) {
        ngp::b200::dataset::NGPDataset::Frame f;
        f.width = f.height = 4;
        f.rgba.assign(64, 255);
        f.focal_x = f.focal_y = 4.0f, f.principal_x = f.principal_y = 2.0f;
        f.camera = {1, 0, 0, 0, 1, 0, 0, 0, 1, 0.5f, 0.5f, 2.0f};
        ds.train = {f, f};
    }
    try {
        ngp::b200::train::InstantNGP model{ds};
        return 0;
    } catch (const std::runtime_error& e) {
        return fail(err, en, e.what());
    }
}

}  // extern "C"
