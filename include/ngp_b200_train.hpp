// C++23 host interface of the library: the reference's `ngp.train` module (ngp.train.ixx:8-53,
// ngp.train.cpp) and `ngp.dataset` types (ngp.dataset.ixx:7-22), as a header over the C ABI of
// ngp_b200.h.  A caller of the reference's InstantNGP switches by including this header instead
// of importing the modules: the same class and method names, the same std::expected results and
// error messages, the same statistics, test images (test/test_NNNN.png, target left, render
// right) and safetensors weights file ("instant-ngp-new.weights.v2", byte for byte).
//
// Differences a caller can see: the constructor takes an optional trainer configuration (grid
// levels, features, table size, scale; the reference fixes them at compile time) and throws
// std::runtime_error when the device set-up fails, as the reference's constructor does; PNGs
// are written uncompressed (same pixels).  Weights files are read by comparing their header,
// parsed and re-serialised with sorted keys, against the model's own header.
#pragma once

#include <algorithm>
#include <array>
#include <bit>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <expected>
#include <filesystem>
#include <format>
#include <fstream>
#include <limits>
#include <map>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

#include "ngp_b200.h"

namespace ngp::b200 {

namespace dataset {
inline constexpr float DEFAULT_SCENE_SCALE = 0.33f;

// ngp.dataset.ixx:7-22: frames of one split share their size and intrinsics.
struct NGPDataset final {
    struct Frame {
        std::vector<std::uint8_t> rgba = {};
        std::array<float, 12> camera   = {};
        std::uint32_t width            = 0;
        std::uint32_t height           = 0;
        float focal_x                  = 0.0f;
        float focal_y                  = 0.0f;
        float principal_x              = 0.0f;
        float principal_y              = 0.0f;
    };
    std::vector<Frame> train      = {};
    std::vector<Frame> validation = {};
    std::vector<Frame> test       = {};
    float scene_scale             = 0.0f;
};
}  // namespace dataset

namespace train {

// ngp.train.ixx:8-38.
struct TrainStats final {
    std::uint32_t step                                    = 0u;
    std::uint32_t rays_per_batch                          = 0u;
    std::uint32_t measured_sample_count_before_compaction = 0u;
    std::uint32_t measured_sample_count                   = 0u;
    std::uint32_t density_grid_occupied_cells             = 0u;
    float loss                                            = 0.0f;
    float elapsed_ms                                      = 0.0f;
    float density_grid_update_ms                          = 0.0f;
    float density_grid_occupancy_ratio                    = 0.0f;
};

struct ValidationStats final {
    std::uint32_t step        = 0u;
    std::uint32_t image_count = 0u;
    std::uint64_t pixel_count = 0u;
    float mse                 = 0.0f;
    float psnr                = 0.0f;
    float elapsed_ms          = 0.0f;
};

struct TestStats final {
    std::uint32_t step                   = 0u;
    std::uint32_t image_count            = 0u;
    std::uint32_t comparison_image_count = 0u;
    std::uint64_t pixel_count            = 0u;
    float mse                            = 0.0f;
    float psnr                           = 0.0f;
    float elapsed_ms                     = 0.0f;
    std::filesystem::path output_dir;
};

// ---- file formats (host only) ---------------------------------------------------------------
namespace format {

inline constexpr std::string_view kWeightsFormat = "instant-ngp-new.weights.v2";
inline constexpr std::uint32_t kMlpWidth = 64, kDensityOutputWidth = 16, kDirectionOutputWidth = 16, kNetworkOutputWidth = 16;
inline constexpr std::uint64_t kMaxHeaderBytes = 100ull * 1024ull * 1024ull;

struct Tensor {
    std::string_view name;
    std::uint64_t param_offset, rows, cols;
};

// The six tensors of a weights file in file order, with their offsets in the packed parameter
// vector [MLP | grid] (ngp.train.cpp:244-251, ngp.train.h:58-86).
inline std::array<Tensor, 6> tensors(const ngp_grid_layout& layout) {
    const std::uint64_t grid_width = static_cast<std::uint64_t>(layout.n_levels) * layout.features_per_level;
    const std::uint64_t rgb_in     = kDensityOutputWidth + kDirectionOutputWidth;
    const std::uint64_t d_in = 0, d_out = d_in + kMlpWidth * grid_width, r_in = d_out + kDensityOutputWidth * kMlpWidth;
    const std::uint64_t r_hid = r_in + kMlpWidth * rgb_in, r_out = r_hid + kMlpWidth * kMlpWidth, grid = r_out + kNetworkOutputWidth * kMlpWidth;
    return {{{"density_mlp.input.weight", d_in, kMlpWidth, grid_width},
             {"density_mlp.output.weight", d_out, kDensityOutputWidth, kMlpWidth},
             {"rgb_mlp.input.weight", r_in, kMlpWidth, rgb_in},
             {"rgb_mlp.hidden.weight", r_hid, kMlpWidth, kMlpWidth},
             {"rgb_mlp.output.weight", r_out, kNetworkOutputWidth, kMlpWidth},
             {"hash_grid.params", grid, layout.offsets[layout.n_levels], layout.features_per_level}}};
}

// The whole safetensors header of the model as compact JSON with sorted keys, the form the
// reference's nlohmann::json::dump() writes (ngp.train.cpp:262-291).
inline std::string weights_header(const ngp_grid_layout& layout, float scene_scale) {
    std::string offsets;
    for (std::uint32_t i = 0; i <= layout.n_levels; ++i) offsets += (i ? "," : "") + std::to_string(layout.offsets[i]);
    const std::map<std::string, std::string> meta = {
        {"format", std::string{kWeightsFormat}},
        {"grid_n_levels", std::to_string(layout.n_levels)},
        {"grid_features_per_level", std::to_string(layout.features_per_level)},
        {"grid_base_resolution", std::to_string(layout.base_resolution)},
        {"grid_log2_hashmap_size", std::to_string(layout.log2_hashmap_size)},
        {"mlp_width", std::to_string(kMlpWidth)},
        {"density_hidden_layers", "1"},
        {"rgb_hidden_layers", "2"},
        {"density_output_width", std::to_string(kDensityOutputWidth)},
        {"direction_output_width", std::to_string(kDirectionOutputWidth)},
        {"rgb_input_width", std::to_string(kDensityOutputWidth + kDirectionOutputWidth)},
        {"network_output_width", std::to_string(kNetworkOutputWidth)},
        {"grid_offsets", offsets},
        {"scene_scale", std::format("{:.9g}", scene_scale)},
    };
    std::map<std::string, std::string> top;
    std::string m = "{";
    for (const auto& [k, v] : meta) m += (m.size() > 1 ? "," : "") + std::format("\"{}\":\"{}\"", k, v);
    top["__metadata__"] = m + "}";
    std::uint64_t off = 0;
    for (const Tensor& t : tensors(layout)) {
        const std::uint64_t bytes = t.rows * t.cols * sizeof(float);
        top[std::string{t.name}]  = std::format("{{\"data_offsets\":[{},{}],\"dtype\":\"F32\",\"shape\":[{},{}]}}", off, off + bytes, t.rows, t.cols);
        off += bytes;
    }
    std::string out = "{";
    for (const auto& [k, v] : top) out += (out.size() > 1 ? "," : "") + std::format("\"{}\":{}", k, v);
    return out + "}";
}

// Minimal JSON reader for safetensors headers (objects, arrays, strings without escapes other
// than \" and \\, unsigned integers); returns the value re-serialised compactly with sorted keys.
class JsonCanon {
public:
    explicit JsonCanon(std::string_view s) : s_(s) {}
    std::string canonical() {
        std::string v = value();
        ws();
        if (i_ != s_.size()) throw std::runtime_error{"safetensors header has trailing characters."};
        return v;
    }

private:
    std::string_view s_;
    std::size_t i_ = 0;
    void ws() {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
    }
    char peek() {
        ws();
        if (i_ >= s_.size()) throw std::runtime_error{"safetensors header ends early."};
        return s_[i_];
    }
    void expect(char c) {
        if (peek() != c) throw std::runtime_error{"safetensors header is not valid JSON."};
        ++i_;
    }
    std::string string() {
        expect('"');
        std::string out = "\"";
        while (i_ < s_.size() && s_[i_] != '"') {
            if (s_[i_] == '\\') {
                if (i_ + 1 >= s_.size() || (s_[i_ + 1] != '"' && s_[i_ + 1] != '\\'))
                    throw std::runtime_error{"safetensors header uses an unsupported escape."};
                out += s_[i_], out += s_[i_ + 1];
                i_ += 2;
                continue;
            }
            out += s_[i_++];
        }
        if (i_ >= s_.size()) throw std::runtime_error{"safetensors header has an unterminated string."};
        ++i_;
        return out + "\"";
    }
    std::string value() {
        const char c = peek();
        if (c == '{') {
            ++i_;
            std::map<std::string, std::string> members;
            if (peek() != '}') {
                for (;;) {
                    std::string key = string();
                    expect(':');
                    if (!members.emplace(key, value()).second) throw std::runtime_error{"safetensors header repeats a key."};
                    if (peek() == ',') {
                        ++i_;
                        continue;
                    }
                    break;
                }
            }
            expect('}');
            std::string out = "{";
            for (const auto& [k, v] : members) out += (out.size() > 1 ? "," : "") + k + ":" + v;
            return out + "}";
        }
        if (c == '[') {
            ++i_;
            std::string out = "[";
            if (peek() != ']') {
                for (;;) {
                    out += (out.size() > 1 ? "," : "") + value();
                    if (peek() == ',') {
                        ++i_;
                        continue;
                    }
                    break;
                }
            }
            expect(']');
            return out + "]";
        }
        if (c == '"') return string();
        if (c >= '0' && c <= '9') {
            const std::size_t b = i_;
            while (i_ < s_.size() && s_[i_] >= '0' && s_[i_] <= '9') ++i_;
            std::string_view digits = s_.substr(b, i_ - b);
            if (digits.size() > 1 && digits[0] == '0') throw std::runtime_error{"safetensors header is not valid JSON."};
            return std::string{digits};
        }
        throw std::runtime_error{"safetensors header holds an unsupported JSON value."};
    }
};

// Write the packed fp32 parameters [MLP | grid] as a weights file (ngp.train.cpp:231-296).
inline void write_weights(const std::filesystem::path& path, const float* params, const ngp_grid_layout& layout, float scene_scale) {
    static_assert(std::endian::native == std::endian::little);
    if (path.empty()) throw std::runtime_error{"weights export path must not be empty."};
    if (!path.parent_path().empty() && !std::filesystem::is_directory(path.parent_path()))
        throw std::runtime_error{std::format("weights export parent directory '{}' does not exist.", path.parent_path().string())};
    const std::string header  = weights_header(layout, scene_scale);
    const std::uint64_t hsize = header.size();
    std::ofstream out{path, std::ios::binary | std::ios::trunc};
    if (!out) throw std::runtime_error{std::format("failed to open weights export path '{}'.", path.string())};
    out.write(reinterpret_cast<const char*>(&hsize), sizeof(hsize));
    out.write(header.data(), static_cast<std::streamsize>(header.size()));
    for (const Tensor& t : tensors(layout))
        out.write(reinterpret_cast<const char*>(params + t.param_offset), static_cast<std::streamsize>(t.rows * t.cols * sizeof(float)));
    if (!out) throw std::runtime_error{std::format("failed to write weights file '{}'.", path.string())};
}

// Read and check a weights file against the model; returns the packed fp32 parameters
// (ngp.train.cpp:298-425: header within 100 MiB, header and metadata equal to the model's,
// data size equal to the tensors, every value finite).
inline std::vector<float> read_weights(const std::filesystem::path& path, const ngp_grid_layout& layout, float scene_scale) {
    static_assert(std::endian::native == std::endian::little);
    if (path.empty()) throw std::runtime_error{"weights load path must not be empty."};
    if (!std::filesystem::is_regular_file(path)) throw std::runtime_error{std::format("weights file '{}' does not exist.", path.string())};
    std::ifstream in{path, std::ios::binary};
    if (!in) throw std::runtime_error{std::format("failed to open weights file '{}'.", path.string())};
    std::vector<char> raw((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
    if (raw.size() < 8) throw std::runtime_error{"weights file is too small for a safetensors header."};
    std::uint64_t hsize = 0;
    std::memcpy(&hsize, raw.data(), sizeof(hsize));
    if (hsize == 0 || hsize > kMaxHeaderBytes) throw std::runtime_error{"invalid safetensors header length."};
    if (8 + hsize > raw.size()) throw std::runtime_error{"safetensors header length exceeds file size."};
    const std::string_view text{raw.data() + 8, static_cast<std::size_t>(hsize)};
    if (text.empty() || text.front() != '{') throw std::runtime_error{"safetensors header must begin with '{'."};
    if (JsonCanon{text}.canonical() != weights_header(layout, scene_scale))
        throw std::runtime_error{"safetensors header does not match the current InstantNGP configuration."};
    const auto ts       = tensors(layout);
    std::uint64_t total = 0, params = 0;
    for (const Tensor& t : ts) total += t.rows * t.cols * sizeof(float), params = std::max(params, t.param_offset + t.rows * t.cols);
    if (raw.size() - 8 - hsize != total) throw std::runtime_error{"safetensors data buffer size does not match tensor offsets."};
    std::vector<float> out(params);
    const char* data = raw.data() + 8 + hsize;
    for (const Tensor& t : ts) {
        std::memcpy(out.data() + t.param_offset, data, t.rows * t.cols * sizeof(float));
        data += t.rows * t.cols * sizeof(float);
    }
    for (float v : out)
        if (!std::isfinite(v)) throw std::runtime_error{"weights file contains non-finite values."};
    return out;
}

// PNG of 8-bit RGB rows, zlib stream of stored (uncompressed) blocks.
inline void write_png(const std::filesystem::path& path, const std::uint8_t* rgb, std::uint32_t width, std::uint32_t height) {
    std::array<std::uint32_t, 256> crc_table{};
    for (std::uint32_t n = 0; n < 256; ++n) {
        std::uint32_t c = n;
        for (int k = 0; k < 8; ++k) c = (c & 1u) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
        crc_table[n] = c;
    }
    auto be32 = [](std::vector<std::uint8_t>& v, std::uint32_t x) {
        v.push_back(static_cast<std::uint8_t>(x >> 24)), v.push_back(static_cast<std::uint8_t>(x >> 16)),
            v.push_back(static_cast<std::uint8_t>(x >> 8)), v.push_back(static_cast<std::uint8_t>(x));
    };
    std::vector<std::uint8_t> file = {0x89, 'P', 'N', 'G', '\r', '\n', 0x1A, '\n'};
    auto chunk = [&](const char* type, const std::vector<std::uint8_t>& body) {
        be32(file, static_cast<std::uint32_t>(body.size()));
        std::uint32_t crc  = 0xFFFFFFFFu;
        auto put           = [&](std::uint8_t b) {
            file.push_back(b);
            crc = crc_table[(crc ^ b) & 0xFFu] ^ (crc >> 8);
        };
        for (int k = 0; k < 4; ++k) put(static_cast<std::uint8_t>(type[k]));
        for (std::uint8_t b : body) put(b);
        be32(file, crc ^ 0xFFFFFFFFu);
    };
    std::vector<std::uint8_t> ihdr;
    be32(ihdr, width), be32(ihdr, height);
    ihdr.insert(ihdr.end(), {8, 2, 0, 0, 0});  // 8-bit RGB, deflate, adaptive filters, no interlace
    chunk("IHDR", ihdr);
    std::vector<std::uint8_t> raw;
    const std::size_t row = static_cast<std::size_t>(width) * 3u;
    raw.reserve((row + 1) * height);
    for (std::uint32_t y = 0; y < height; ++y) {
        raw.push_back(0);  // filter: none
        raw.insert(raw.end(), rgb + y * row, rgb + (y + 1) * row);
    }
    std::vector<std::uint8_t> z = {0x78, 0x01};
    std::uint32_t a = 1, b = 0;
    for (std::uint8_t v : raw) a = (a + v) % 65521u, b = (b + a) % 65521u;
    std::size_t off = 0;
    do {  // stored blocks of at most 65535 bytes; the last one has BFINAL set
        const std::size_t n = std::min<std::size_t>(65535, raw.size() - off);
        const auto len      = static_cast<std::uint16_t>(n);
        const auto nlen     = static_cast<std::uint16_t>(~len);
        z.push_back(off + n >= raw.size() ? 1 : 0);
        z.push_back(static_cast<std::uint8_t>(len)), z.push_back(static_cast<std::uint8_t>(len >> 8));
        z.push_back(static_cast<std::uint8_t>(nlen)), z.push_back(static_cast<std::uint8_t>(nlen >> 8));
        z.insert(z.end(), raw.begin() + static_cast<std::ptrdiff_t>(off), raw.begin() + static_cast<std::ptrdiff_t>(off + n));
        off += n;
    } while (off < raw.size());
    be32(z, (b << 16) | a);
    chunk("IDAT", z);
    chunk("IEND", {});
    std::ofstream out{path, std::ios::binary | std::ios::trunc};
    out.write(reinterpret_cast<const char*>(file.data()), static_cast<std::streamsize>(file.size()));
    if (!out) throw std::runtime_error{std::format("failed to write test comparison image '{}'.", path.string())};
}

}  // namespace format

// ngp.train.ixx:40-53 over the C ABI trainer.
class InstantNGP final {
public:
    explicit InstantNGP(const dataset::NGPDataset& dataset, const ngp_trainer_config* config = nullptr) : scene_scale_(dataset.scene_scale) {
        ngp_trainer_config cfg{};
        if (config != nullptr) cfg = *config;
        else ngp_trainer_default_config(&cfg);
        check(ngp_grid_layout_make(cfg.n_levels, cfg.features_per_level, cfg.log2_hashmap_size, cfg.base_resolution, cfg.log2_per_level_scale, &layout_));
        pack(dataset.train, "train", train_);
        pack(dataset.validation, "validation", validation_);
        pack(dataset.test, "test", test_);
        if (train_.split.frame_count == 0) throw std::runtime_error{"the dataset has no training images."};
        check(ngp_trainer_create(&cfg, &train_.split, validation_.split.frame_count ? &validation_.split : nullptr,
                                 test_.split.frame_count ? &test_.split : nullptr, &handle_));
        // the trainer keeps its own device copies of the splits; only their shapes stay here
        for (PackedSplit* p : {&train_, &validation_, &test_}) p->storage = {}, p->split.pixels = nullptr, p->split.camera = nullptr;
    }
    ~InstantNGP() noexcept { ngp_trainer_destroy(handle_); }
    InstantNGP(const InstantNGP&)                = delete;
    InstantNGP& operator=(const InstantNGP&)     = delete;
    InstantNGP(InstantNGP&&) noexcept            = delete;
    InstantNGP& operator=(InstantNGP&&) noexcept = delete;

    std::expected<TrainStats, std::string> train(std::int32_t iters) {
        try {
            const auto start = std::chrono::steady_clock::now();
            ngp_train_stats s{};
            check(ngp_trainer_train(handle_, iters, &s));
            step_ = s.step;
            return TrainStats{
                .step                                    = s.step,
                .rays_per_batch                          = s.rays_per_batch,
                .measured_sample_count_before_compaction = s.measured_sample_count_before_compaction,
                .measured_sample_count                   = s.measured_sample_count,
                .density_grid_occupied_cells             = s.density_grid_occupied_cells,
                .loss                                    = s.loss,
                .elapsed_ms                              = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - start).count(),
                .density_grid_update_ms                  = s.density_grid_update_ms,
                .density_grid_occupancy_ratio            = s.density_grid_occupancy_ratio,
            };
        } catch (const std::exception& error) {
            return std::unexpected{std::string{error.what()}};
        }
    }

    std::expected<ValidationStats, std::string> validate() const {
        try {
            const std::uint32_t frames = validation_.split.frame_count;
            if (frames == 0u) throw std::runtime_error{"No validation images are available in the current dataset."};
            const auto start = std::chrono::steady_clock::now();
            double sse       = 0.0;
            std::uint64_t px = 0;
            check(ngp_trainer_evaluate(handle_, 1, 0, frames, nullptr, &sse, &px));
            const double mse = sse / (static_cast<double>(px) * 3.0);
            if (!std::isfinite(mse)) throw std::runtime_error{"validation produced non-finite MSE."};
            return ValidationStats{
                .step        = step_,
                .image_count = frames,
                .pixel_count = px,
                .mse         = static_cast<float>(mse),
                .psnr        = psnr(mse),
                .elapsed_ms  = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - start).count(),
            };
        } catch (const std::exception& error) {
            return std::unexpected{std::string{error.what()}};
        }
    }

    // Test PSNR and one comparison PNG per test image in `output_dir` ("test", as the reference).
    std::expected<TestStats, std::string> test(const std::filesystem::path& output_dir = "test") const {
        try {
            const ngp_split& s = test_.split;
            if (s.frame_count == 0u) throw std::runtime_error{"No test images are available in the current dataset."};
            if (output_dir.empty()) throw std::runtime_error{"test output directory must not be empty."};
            if (std::filesystem::exists(output_dir) && !std::filesystem::is_directory(output_dir))
                throw std::runtime_error{std::format("test output path '{}' is not a directory.", output_dir.string())};
            std::filesystem::create_directories(output_dir);
            const auto start = std::chrono::steady_clock::now();
            std::vector<std::uint8_t> comparison(static_cast<std::size_t>(s.width) * s.height * 6u);
            double sse_total      = 0.0;
            std::uint64_t px_total = 0;
            for (std::uint32_t i = 0; i < s.frame_count; ++i) {
                double sse       = 0.0;
                std::uint64_t px = 0;
                check(ngp_trainer_evaluate(handle_, 2, i, 1, comparison.data(), &sse, &px));
                sse_total += sse, px_total += px;
                format::write_png(output_dir / std::format("test_{:04}.png", i), comparison.data(), s.width * 2u, s.height);
            }
            const double mse = sse_total / (static_cast<double>(px_total) * 3.0);
            if (!std::isfinite(mse)) throw std::runtime_error{"test produced non-finite MSE."};
            return TestStats{
                .step                   = step_,
                .image_count            = s.frame_count,
                .comparison_image_count = s.frame_count,
                .pixel_count            = px_total,
                .mse                    = static_cast<float>(mse),
                .psnr                   = psnr(mse),
                .elapsed_ms             = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - start).count(),
                .output_dir             = output_dir,
            };
        } catch (const std::exception& error) {
            return std::unexpected{std::string{error.what()}};
        }
    }

    std::expected<void, std::string> export_weights(const std::filesystem::path& path) const {
        try {
            std::vector<float> params(ngp_trainer_param_count(handle_));
            check(ngp_trainer_get_params(handle_, params.data(), static_cast<std::uint32_t>(params.size())));
            format::write_weights(path, params.data(), layout_, scene_scale_);
            return {};
        } catch (const std::exception& error) {
            return std::unexpected{std::string{error.what()}};
        }
    }

    std::expected<void, std::string> load_weights(const std::filesystem::path& path) {
        try {
            if (step_ != 0u) throw std::runtime_error{"weights can only be loaded before training starts."};
            std::vector<float> params = format::read_weights(path, layout_, scene_scale_);
            if (params.size() != ngp_trainer_param_count(handle_)) throw std::runtime_error{"weights file does not match the model's parameter count."};
            check(ngp_trainer_set_params(handle_, params.data(), static_cast<std::uint32_t>(params.size())));
            return {};
        } catch (const std::exception& error) {
            return std::unexpected{std::string{error.what()}};
        }
    }

    // The C ABI handle, for the library's other trainer entry points (rendering, profiling).
    ngp_trainer* handle() const { return handle_; }

private:
    struct PackedSplit {
        ngp_split split{};
        std::vector<std::uint8_t> storage;  // pixels, then cameras (kept until the trainer copied them)
    };

    static void check(int status) {
        if (status != NGP_OK) throw std::runtime_error{ngp_last_error()};
    }
    static float psnr(double mse) { return mse > 0.0 ? static_cast<float>(-10.0 * std::log10(mse)) : std::numeric_limits<float>::infinity(); }

    // Contiguous [frames][h][w][4] pixels and [frames][12] cameras of one split.
    static void pack(const std::vector<dataset::NGPDataset::Frame>& frames, const char* name, PackedSplit& out) {
        out = PackedSplit{};
        if (frames.empty()) return;
        const auto& f0 = frames.front();
        for (const auto& f : frames) {
            if (f.width != f0.width || f.height != f0.height || f.focal_x != f0.focal_x || f.focal_y != f0.focal_y || f.principal_x != f0.principal_x ||
                f.principal_y != f0.principal_y)
                throw std::runtime_error{std::format("{} frames must share their size and intrinsics.", name)};
            if (f.rgba.size() != static_cast<std::size_t>(f.width) * f.height * 4u)
                throw std::runtime_error{std::format("{} frame pixel buffer has the wrong size.", name)};
        }
        const std::size_t px = static_cast<std::size_t>(f0.width) * f0.height * 4u;
        const std::size_t pix_bytes = px * frames.size(), cam_bytes = frames.size() * 12u * sizeof(float);
        out.storage.resize(pix_bytes + cam_bytes + alignof(float));
        std::uint8_t* pix = out.storage.data();
        auto* cam         = reinterpret_cast<float*>(out.storage.data() + ((pix_bytes + alignof(float) - 1) / alignof(float)) * alignof(float));
        for (std::size_t i = 0; i < frames.size(); ++i) {
            std::memcpy(pix + i * px, frames[i].rgba.data(), px);
            std::memcpy(cam + i * 12u, frames[i].camera.data(), 12u * sizeof(float));
        }
        out.split = ngp_split{pix, cam, static_cast<std::uint32_t>(frames.size()), f0.width, f0.height, f0.focal_x, f0.focal_y, f0.principal_x,
                              f0.principal_y};
    }

    ngp_trainer* handle_ = nullptr;
    ngp_grid_layout layout_{};
    float scene_scale_  = 0.0f;
    std::uint32_t step_ = 0u;
    PackedSplit train_, validation_, test_;
};

}  // namespace train
}  // namespace ngp::b200

// The reference's callers name these types ngp::train::InstantNGP and ngp::dataset::NGPDataset
// (ngp.train.ixx:40, ngp.dataset.ixx:7): the aliases let that code compile unchanged.  Define
// NGP_B200_NO_REFERENCE_NAMES to leave them out (e.g. beside the reference's own modules).
#ifndef NGP_B200_NO_REFERENCE_NAMES
namespace ngp {
namespace train   = ngp::b200::train;
namespace dataset = ngp::b200::dataset;
}  // namespace ngp
#endif
