// C++23 scene loaders of the reference's `ngp.dataset` module (ngp.dataset.ixx:24-25,
// ngp.dataset.cpp:12-190) for the C++ host interface (ngp_b200_train.hpp): NeRF-synthetic
// (transforms_{train,val,test}.json + images) and DD-NeRF (cameras.json + images/, split by the
// FNV-1a hash of each file name).  Header only, no third-party code: a JSON reader (comments
// allowed, as the reference parses), and a PNG decoder (zlib inflate, scanline filters) for
// 8-bit, non-interlaced PNGs of every colour type, expanded to RGBA8 as the reference's
// stbi_load(..., 4) does.  Cameras are converted in float32, one rounding per operation: columns
// 1 and 2 negated, the position scaled by the scene scale and offset by 0.5, the axes permuted
// (x, y, z) -> (y, z, x) into three axis columns and the origin.
#pragma once

#include <array>
#include <charconv>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <expected>
#include <filesystem>
#include <format>
#include <fstream>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

#include "ngp_b200_train.hpp"

namespace ngp::b200::dataset {

namespace detail {

// ---- JSON ------------------------------------------------------------------------------------
struct Json {
    enum class Kind { Null, Bool, Number, String, Array, Object } kind = Kind::Null;
    bool boolean  = false;
    double number = 0.0;
    std::string text;
    std::vector<Json> items;
    std::vector<std::pair<std::string, Json>> members;

    const Json& at(std::string_view key) const {
        if (kind != Kind::Object) throw std::runtime_error{std::format("JSON value is not an object (looking up '{}').", key)};
        for (const auto& [k, v] : members)
            if (k == key) return v;
        throw std::runtime_error{std::format("JSON key '{}' not found.", key)};
    }
    const Json& at(std::size_t i) const {
        if (kind != Kind::Array) throw std::runtime_error{"JSON value is not an array."};
        if (i >= items.size()) throw std::runtime_error{"JSON array index out of range."};
        return items[i];
    }
    bool contains(std::string_view key) const {
        if (kind != Kind::Object) return false;
        for (const auto& m : members)
            if (m.first == key) return true;
        return false;
    }
    double as_number() const {
        if (kind != Kind::Number) throw std::runtime_error{"JSON value is not a number."};
        return number;
    }
    float as_float() const { return static_cast<float>(as_number()); }
    std::uint32_t as_u32() const {
        const double v = as_number();
        if (!(v >= 0.0) || v > 4294967295.0 || v != std::floor(v)) throw std::runtime_error{"JSON value is not an unsigned 32-bit integer."};
        return static_cast<std::uint32_t>(v);
    }
    const std::string& as_string() const {
        if (kind != Kind::String) throw std::runtime_error{"JSON value is not a string."};
        return text;
    }
};

class JsonParser {
public:
    explicit JsonParser(std::string_view s) : s_(s) {}
    Json parse() {
        Json v = value();
        skip();
        if (i_ != s_.size()) fail("trailing characters");
        return v;
    }

private:
    std::string_view s_;
    std::size_t i_ = 0;

    [[noreturn]] void fail(const char* what) const { throw std::runtime_error{std::format("JSON parse error at byte {}: {}.", i_, what)}; }
    void skip() {  // whitespace and comments
        for (;;) {
            while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t')) ++i_;
            if (i_ + 1 < s_.size() && s_[i_] == '/' && s_[i_ + 1] == '/') {
                while (i_ < s_.size() && s_[i_] != '\n') ++i_;
            } else if (i_ + 1 < s_.size() && s_[i_] == '/' && s_[i_ + 1] == '*') {
                const std::size_t end = s_.find("*/", i_ + 2);
                if (end == std::string_view::npos) fail("unterminated comment");
                i_ = end + 2;
            } else {
                return;
            }
        }
    }
    char peek() {
        skip();
        if (i_ >= s_.size()) fail("unexpected end");
        return s_[i_];
    }
    void expect(char c) {
        if (peek() != c) fail("unexpected character");
        ++i_;
    }
    static void utf8(std::string& out, std::uint32_t cp) {
        if (cp < 0x80) {
            out += static_cast<char>(cp);
        } else if (cp < 0x800) {
            out += static_cast<char>(0xC0 | (cp >> 6)), out += static_cast<char>(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += static_cast<char>(0xE0 | (cp >> 12)), out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F)), out += static_cast<char>(0x80 | (cp & 0x3F));
        } else {
            out += static_cast<char>(0xF0 | (cp >> 18)), out += static_cast<char>(0x80 | ((cp >> 12) & 0x3F));
            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F)), out += static_cast<char>(0x80 | (cp & 0x3F));
        }
    }
    std::uint32_t hex4() {
        if (i_ + 4 > s_.size()) fail("short \\u escape");
        std::uint32_t v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = s_[i_++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= static_cast<std::uint32_t>(c - '0');
            else if (c >= 'a' && c <= 'f') v |= static_cast<std::uint32_t>(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= static_cast<std::uint32_t>(c - 'A' + 10);
            else fail("bad \\u escape");
        }
        return v;
    }
    std::string string() {
        expect('"');
        std::string out;
        for (;;) {
            if (i_ >= s_.size()) fail("unterminated string");
            const char c = s_[i_++];
            if (c == '"') return out;
            if (c != '\\') {
                out += c;
                continue;
            }
            if (i_ >= s_.size()) fail("unterminated escape");
            const char e = s_[i_++];
            switch (e) {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'n': out += '\n'; break;
                case 'r': out += '\r'; break;
                case 't': out += '\t'; break;
                case 'u': {
                    std::uint32_t cp = hex4();
                    if (cp >= 0xD800 && cp < 0xDC00 && i_ + 1 < s_.size() && s_[i_] == '\\' && s_[i_ + 1] == 'u') {
                        i_ += 2;
                        const std::uint32_t lo = hex4();
                        if (lo < 0xDC00 || lo >= 0xE000) fail("bad surrogate pair");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    }
                    utf8(out, cp);
                    break;
                }
                default: fail("bad escape");
            }
        }
    }
    Json value() {
        Json v;
        const char c = peek();
        if (c == '{') {
            ++i_;
            v.kind = Json::Kind::Object;
            if (peek() == '}') return ++i_, v;
            for (;;) {
                std::string key = string();
                expect(':');
                v.members.emplace_back(std::move(key), value());
                if (peek() == ',') {
                    ++i_;
                    continue;
                }
                expect('}');
                return v;
            }
        }
        if (c == '[') {
            ++i_;
            v.kind = Json::Kind::Array;
            if (peek() == ']') return ++i_, v;
            for (;;) {
                v.items.push_back(value());
                if (peek() == ',') {
                    ++i_;
                    continue;
                }
                expect(']');
                return v;
            }
        }
        if (c == '"') {
            v.kind = Json::Kind::String;
            v.text = string();
            return v;
        }
        if (s_.substr(i_, 4) == "true") return i_ += 4, v.kind = Json::Kind::Bool, v.boolean = true, v;
        if (s_.substr(i_, 5) == "false") return i_ += 5, v.kind = Json::Kind::Bool, v;
        if (s_.substr(i_, 4) == "null") return i_ += 4, v;
        v.kind              = Json::Kind::Number;
        const char* first   = s_.data() + i_;
        const auto [ptr, ec] = std::from_chars(first, s_.data() + s_.size(), v.number);
        if (ec != std::errc{} || ptr == first) fail("bad number");
        i_ += static_cast<std::size_t>(ptr - first);
        return v;
    }
};

inline Json read_json(const std::filesystem::path& path) {
    std::ifstream in{path, std::ios::binary};
    if (!in) throw std::runtime_error{std::format("failed to open '{}'.", path.string())};
    const std::string text((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
    return JsonParser{text}.parse();
}

// ---- zlib inflate (RFC 1950 / 1951) ----------------------------------------------------------
class Inflater {
public:
    Inflater(const std::uint8_t* data, std::size_t size) : p_(data), n_(size) {}

    std::vector<std::uint8_t> run(std::size_t size_hint) {
        if (n_ < 2) throw std::runtime_error{"zlib stream too short."};
        const std::uint32_t cmf = p_[0], flg = p_[1];
        if ((cmf & 0x0F) != 8 || ((cmf << 8) | flg) % 31 != 0 || (flg & 0x20)) throw std::runtime_error{"unsupported zlib stream."};
        pos_ = 2;
        out_.reserve(size_hint);
        bool last = false;
        while (!last) {
            last             = bits(1) != 0;
            const auto btype = bits(2);
            if (btype == 0) stored();
            else if (btype == 1) fixed();
            else if (btype == 2) dynamic();
            else throw std::runtime_error{"invalid deflate block type."};
        }
        return std::move(out_);
    }

private:
    struct Huffman {
        std::array<std::uint16_t, 16> count{};
        std::vector<std::uint16_t> symbol;
    };

    const std::uint8_t* p_;
    std::size_t n_, pos_ = 0;
    std::uint32_t bitbuf_ = 0, bitcnt_ = 0;
    std::vector<std::uint8_t> out_;

    std::uint32_t bits(std::uint32_t need) {
        while (bitcnt_ < need) {
            if (pos_ >= n_) throw std::runtime_error{"deflate stream ends early."};
            bitbuf_ |= static_cast<std::uint32_t>(p_[pos_++]) << bitcnt_;
            bitcnt_ += 8;
        }
        const std::uint32_t v = bitbuf_ & ((1u << need) - 1u);
        bitbuf_ >>= need;
        bitcnt_ -= need;
        return v;
    }
    void stored() {
        bitbuf_ = 0, bitcnt_ = 0;  // to the byte boundary
        if (pos_ + 4 > n_) throw std::runtime_error{"deflate stored block ends early."};
        const std::uint32_t len = p_[pos_] | (p_[pos_ + 1] << 8), nlen = p_[pos_ + 2] | (p_[pos_ + 3] << 8);
        pos_ += 4;
        if ((len ^ 0xFFFFu) != nlen) throw std::runtime_error{"deflate stored block length check failed."};
        if (pos_ + len > n_) throw std::runtime_error{"deflate stored block ends early."};
        out_.insert(out_.end(), p_ + pos_, p_ + pos_ + len);
        pos_ += len;
    }
    // Canonical Huffman code from code lengths (RFC 1951 3.2.2).
    static Huffman build(const std::uint8_t* lengths, std::size_t n) {
        Huffman h;
        h.symbol.assign(n, 0);
        for (std::size_t s = 0; s < n; ++s) ++h.count[lengths[s]];
        h.count[0] = 0;
        std::array<std::uint16_t, 16> offs{};
        int left = 1;
        for (int len = 1; len < 16; ++len) {
            left = (left << 1) - h.count[len];
            if (left < 0) throw std::runtime_error{"over-subscribed Huffman code."};
            offs[len] = static_cast<std::uint16_t>((len == 1 ? 0 : offs[len - 1]) + (len == 1 ? 0 : h.count[len - 1]));
        }
        for (std::size_t s = 0; s < n; ++s)
            if (lengths[s]) h.symbol[offs[lengths[s]]++] = static_cast<std::uint16_t>(s);
        return h;
    }
    std::uint32_t decode(const Huffman& h) {
        int code = 0, first = 0, index = 0;
        for (int len = 1; len < 16; ++len) {
            code |= static_cast<int>(bits(1));
            const int count = h.count[len];
            if (code - count < first) return h.symbol[static_cast<std::size_t>(index + (code - first))];
            index += count;
            first += count;
            first <<= 1;
            code <<= 1;
        }
        throw std::runtime_error{"invalid Huffman code."};
    }
    void codes(const Huffman& lit, const Huffman& dist) {
        static constexpr std::array<std::uint16_t, 29> len_base = {3,  4,  5,  6,  7,  8,  9,  10, 11,  13,  15,  17,  19,  23, 27,
                                                                   31, 35, 43, 51, 59, 67, 83, 99, 115, 131, 163, 195, 227, 258};
        static constexpr std::array<std::uint8_t, 29> len_extra = {0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 2, 3, 3, 3, 3, 4, 4, 4, 4, 5, 5, 5, 5, 0};
        static constexpr std::array<std::uint16_t, 30> dist_base = {1,   2,   3,   4,   5,   7,    9,    13,   17,   25,   33,   49,   65,    97,    129,
                                                                    193, 257, 385, 513, 769, 1025, 1537, 2049, 3073, 4097, 6145, 8193, 12289, 16385, 24577};
        static constexpr std::array<std::uint8_t, 30> dist_extra = {0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6, 6, 7, 7, 8, 8, 9, 9, 10, 10, 11, 11, 12, 12, 13, 13};
        for (;;) {
            std::uint32_t sym = decode(lit);
            if (sym < 256) {
                out_.push_back(static_cast<std::uint8_t>(sym));
            } else if (sym == 256) {
                return;
            } else {
                sym -= 257;
                if (sym >= 29) throw std::runtime_error{"invalid deflate length code."};
                const std::size_t len = len_base[sym] + bits(len_extra[sym]);
                const std::uint32_t d = decode(dist);
                if (d >= 30) throw std::runtime_error{"invalid deflate distance code."};
                const std::size_t back = dist_base[d] + bits(dist_extra[d]);
                if (back > out_.size()) throw std::runtime_error{"deflate distance reaches before the output."};
                const std::size_t from = out_.size() - back;
                for (std::size_t k = 0; k < len; ++k) out_.push_back(out_[from + k]);
            }
        }
    }
    void fixed() {
        std::array<std::uint8_t, 288> l{};
        for (int s = 0; s < 144; ++s) l[s] = 8;
        for (int s = 144; s < 256; ++s) l[s] = 9;
        for (int s = 256; s < 280; ++s) l[s] = 7;
        for (int s = 280; s < 288; ++s) l[s] = 8;
        std::array<std::uint8_t, 30> d{};
        d.fill(5);
        codes(build(l.data(), l.size()), build(d.data(), d.size()));
    }
    void dynamic() {
        const std::uint32_t nlen = bits(5) + 257, ndist = bits(5) + 1, ncode = bits(4) + 4;
        if (nlen > 286 || ndist > 30) throw std::runtime_error{"invalid dynamic block header."};
        static constexpr std::array<std::uint8_t, 19> order = {16, 17, 18, 0, 8, 7, 9, 6, 10, 5, 11, 4, 12, 3, 13, 2, 14, 1, 15};
        std::array<std::uint8_t, 19> cl{};
        for (std::uint32_t k = 0; k < ncode; ++k) cl[order[k]] = static_cast<std::uint8_t>(bits(3));
        const Huffman lencode = build(cl.data(), cl.size());
        std::array<std::uint8_t, 316> lengths{};
        for (std::uint32_t k = 0; k < nlen + ndist;) {
            const std::uint32_t sym = decode(lencode);
            if (sym < 16) {
                lengths[k++] = static_cast<std::uint8_t>(sym);
                continue;
            }
            std::uint8_t v = 0;
            std::uint32_t rep = 0;
            if (sym == 16) {
                if (k == 0) throw std::runtime_error{"repeat with no previous length."};
                v = lengths[k - 1], rep = 3 + bits(2);
            } else if (sym == 17) {
                rep = 3 + bits(3);
            } else {
                rep = 11 + bits(7);
            }
            if (k + rep > nlen + ndist) throw std::runtime_error{"too many code lengths."};
            while (rep--) lengths[k++] = v;
        }
        if (lengths[256] == 0) throw std::runtime_error{"no end-of-block code."};
        codes(build(lengths.data(), nlen), build(lengths.data() + nlen, ndist));
    }
};

// ---- PNG (8-bit, non-interlaced) -> RGBA8 ------------------------------------------------------
inline std::vector<std::uint8_t> load_png_rgba(const std::filesystem::path& path, std::uint32_t& width, std::uint32_t& height) {
    std::ifstream in{path, std::ios::binary};
    if (!in) throw std::runtime_error{std::format("failed to load image '{}'.", path.string())};
    const std::vector<std::uint8_t> f((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
    static constexpr std::array<std::uint8_t, 8> sig = {0x89, 'P', 'N', 'G', '\r', '\n', 0x1A, '\n'};
    if (f.size() < 8 || !std::equal(sig.begin(), sig.end(), f.begin())) throw std::runtime_error{std::format("'{}' is not a PNG image.", path.string())};
    auto be32 = [&](std::size_t o) { return (std::uint32_t{f[o]} << 24) | (std::uint32_t{f[o + 1]} << 16) | (std::uint32_t{f[o + 2]} << 8) | f[o + 3]; };
    std::uint32_t depth = 0, ctype = 0, interlace = 0;
    width = height = 0;
    std::vector<std::uint8_t> idat, palette, trns;
    for (std::size_t o = 8; o + 12 <= f.size();) {
        const std::uint32_t len = be32(o);
        const std::string_view type{reinterpret_cast<const char*>(f.data() + o + 4), 4};
        if (o + 12 + static_cast<std::size_t>(len) > f.size()) throw std::runtime_error{std::format("PNG '{}' is truncated.", path.string())};
        const std::uint8_t* body = f.data() + o + 8;
        if (type == "IHDR") {
            if (len < 13) throw std::runtime_error{"bad PNG header."};
            width = be32(o + 8), height = be32(o + 12), depth = body[8], ctype = body[9], interlace = body[12];
        } else if (type == "PLTE") {
            palette.assign(body, body + len);
        } else if (type == "tRNS") {
            trns.assign(body, body + len);
        } else if (type == "IDAT") {
            idat.insert(idat.end(), body, body + len);
        } else if (type == "IEND") {
            break;
        }
        o += 12 + static_cast<std::size_t>(len);
    }
    if (width == 0 || height == 0) throw std::runtime_error{std::format("image '{}' has invalid dimensions.", path.string())};
    const std::uint32_t channels = ctype == 0 ? 1 : ctype == 2 ? 3 : ctype == 3 ? 1 : ctype == 4 ? 2 : ctype == 6 ? 4 : 0;
    if (depth != 8 || channels == 0 || interlace != 0)
        throw std::runtime_error{std::format("PNG '{}' is not an 8-bit non-interlaced image (the formats this loader reads).", path.string())};
    if (ctype == 3 && palette.empty()) throw std::runtime_error{"palette PNG without PLTE."};
    const std::size_t stride = static_cast<std::size_t>(width) * channels;
    const std::vector<std::uint8_t> raw = Inflater{idat.data(), idat.size()}.run((stride + 1) * height);
    if (raw.size() < (stride + 1) * height) throw std::runtime_error{std::format("PNG '{}' has too little image data.", path.string())};
    std::vector<std::uint8_t> img(stride * height);
    for (std::uint32_t y = 0; y < height; ++y) {  // scanline filters (PNG spec 9.2)
        const std::uint8_t filter = raw[y * (stride + 1)];
        const std::uint8_t* src   = raw.data() + y * (stride + 1) + 1;
        std::uint8_t* row         = img.data() + y * stride;
        const std::uint8_t* up    = y > 0 ? row - stride : nullptr;
        for (std::size_t x = 0; x < stride; ++x) {
            const int a = x >= channels ? row[x - channels] : 0, b = up ? up[x] : 0, c = (up && x >= channels) ? up[x - channels] : 0;
            int pred = 0;
            switch (filter) {
                case 0: pred = 0; break;
                case 1: pred = a; break;
                case 2: pred = b; break;
                case 3: pred = (a + b) / 2; break;
                case 4: {
                    const int p = a + b - c, pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
                    pred = (pa <= pb && pa <= pc) ? a : (pb <= pc ? b : c);
                    break;
                }
                default: throw std::runtime_error{std::format("PNG '{}' uses an invalid filter.", path.string())};
            }
            row[x] = static_cast<std::uint8_t>(src[x] + pred);
        }
    }
    std::vector<std::uint8_t> rgba(static_cast<std::size_t>(width) * height * 4u);
    for (std::size_t i = 0; i < static_cast<std::size_t>(width) * height; ++i) {
        const std::uint8_t* s = img.data() + i * channels;
        std::uint8_t* d       = rgba.data() + i * 4u;
        switch (ctype) {
            case 0:
                d[0] = d[1] = d[2] = s[0];
                d[3] = (trns.size() >= 2 && s[0] == trns[1]) ? 0 : 255;
                break;
            case 2:
                d[0] = s[0], d[1] = s[1], d[2] = s[2];
                d[3] = (trns.size() >= 6 && s[0] == trns[1] && s[1] == trns[3] && s[2] == trns[5]) ? 0 : 255;
                break;
            case 3: {
                const std::size_t k = s[0];
                if (3 * k + 2 >= palette.size()) throw std::runtime_error{std::format("PNG '{}' indexes past its palette.", path.string())};
                d[0] = palette[3 * k], d[1] = palette[3 * k + 1], d[2] = palette[3 * k + 2];
                d[3] = k < trns.size() ? trns[k] : 255;
                break;
            }
            case 4: d[0] = d[1] = d[2] = s[0], d[3] = s[1]; break;
            default: std::memcpy(d, s, 4); break;
        }
    }
    return rgba;
}

// ---- cameras ---------------------------------------------------------------------------------
inline float mul_rn(float a, float b) {
    volatile float r = a * b;  // one rounding; not contracted with the following addition
    return r;
}

// 12-float camera of one frame (ngp.dataset.cpp:47-65).
inline std::array<float, 12> ngp_camera(const Json& transform_matrix, float scene_scale) {
    float cam[4][4];  // [column][row]
    for (std::size_t row = 0; row < 4; ++row)
        for (std::size_t col = 0; col < 4; ++col) cam[col][row] = transform_matrix.at(row).at(col).as_float();
    for (std::size_t r = 0; r < 4; ++r) cam[1][r] = -cam[1][r], cam[2][r] = -cam[2][r];
    for (std::size_t r = 0; r < 3; ++r) cam[3][r] = mul_rn(cam[3][r], scene_scale) + 0.5f;
    return {cam[0][1], cam[0][2], cam[0][0], cam[1][1], cam[1][2], cam[1][0], cam[2][1], cam[2][2], cam[2][0], cam[3][1], cam[3][2], cam[3][0]};
}

inline std::filesystem::path frame_path(const std::filesystem::path& root, const std::string& file, bool default_png) {
    std::filesystem::path p = file;
    p.make_preferred();
    if (default_png && p.extension().empty()) p.replace_extension(".png");
    if (p.is_relative()) p = root / p;
    return p.lexically_normal();
}

inline std::vector<NGPDataset::Frame> nerf_synthetic_split(const std::filesystem::path& root, std::string_view file_name, float scene_scale) {
    const std::filesystem::path json_path = root / file_name;
    const Json json                       = read_json(json_path);
    const float angle                     = json.at("camera_angle_x").as_float();
    const Json& frames_json               = json.at("frames");
    std::vector<NGPDataset::Frame> frames;
    for (const Json& fj : frames_json.items) {
        const std::filesystem::path image = frame_path(json_path.parent_path(), fj.at("file_path").as_string(), true);
        NGPDataset::Frame f;
        f.rgba   = load_png_rgba(image, f.width, f.height);
        f.camera = ngp_camera(fj.at("transform_matrix"), scene_scale);
        // focal = 0.5 w / tan(angle / 2): the tangent rounded to float32 from double precision
        const float half_w = 0.5f * static_cast<float>(f.width);
        f.focal_x = f.focal_y = half_w / static_cast<float>(std::tan(static_cast<double>(angle * 0.5f)));
        f.principal_x         = static_cast<float>(f.width) * 0.5f;
        f.principal_y         = static_cast<float>(f.height) * 0.5f;
        frames.push_back(std::move(f));
    }
    return frames;
}

}  // namespace detail

// transforms_{train,val,test}.json + images (ngp.dataset.cpp:12-93).
inline std::expected<NGPDataset, std::string> load_nerf_synthetic(const std::filesystem::path& path, float scene_scale = DEFAULT_SCENE_SCALE) {
    try {
        if (!std::isfinite(scene_scale) || scene_scale <= 0.0f) throw std::runtime_error{"scene scale must be finite and positive."};
        NGPDataset ds;
        ds.train       = detail::nerf_synthetic_split(path, "transforms_train.json", scene_scale);
        ds.validation  = detail::nerf_synthetic_split(path, "transforms_val.json", scene_scale);
        ds.test        = detail::nerf_synthetic_split(path, "transforms_test.json", scene_scale);
        ds.scene_scale = scene_scale;
        return ds;
    } catch (const std::exception& error) {
        return std::unexpected{std::string{error.what()}};
    }
}

// cameras.json + images/, frames split by FNV-1a of the file name: % 10 == 0 test, == 1
// validation, otherwise train (ngp.dataset.cpp:96-190).
inline std::expected<NGPDataset, std::string> load_dd_nerf_dataset(const std::filesystem::path& path, float scene_scale = DEFAULT_SCENE_SCALE) {
    using detail::Json;
    try {
        if (!std::isfinite(scene_scale) || scene_scale <= 0.0f) throw std::runtime_error{"scene scale must be finite and positive."};
        const std::filesystem::path json_path = path / "cameras.json";
        if (!std::filesystem::is_regular_file(json_path)) throw std::runtime_error{std::format("DD-NeRF dataset '{}' is missing cameras.json.", path.string())};
        if (!std::filesystem::is_directory(path / "images"))
            throw std::runtime_error{std::format("DD-NeRF dataset '{}' is missing an images directory.", path.string())};
        const Json json         = detail::read_json(json_path);
        const Json& frames_json = json.at("frames");
        const std::uint32_t w = json.at("w").as_u32(), h = json.at("h").as_u32();
        const float fx = json.at("fl_x").as_float(), fy = json.at("fl_y").as_float(), cx = json.at("cx").as_float(), cy = json.at("cy").as_float();
        if (frames_json.kind != Json::Kind::Array || frames_json.items.empty())
            throw std::runtime_error{"DD-NeRF cameras.json must contain a non-empty frames array."};
        if (w == 0u || h == 0u) throw std::runtime_error{"DD-NeRF cameras.json declares invalid image dimensions."};
        if (!std::isfinite(fx) || !std::isfinite(fy) || fx <= 0.0f || fy <= 0.0f) throw std::runtime_error{"DD-NeRF cameras.json declares invalid focal lengths."};
        if (!std::isfinite(cx) || !std::isfinite(cy) || cx < 0.0f || cy < 0.0f || cx >= static_cast<float>(w) || cy >= static_cast<float>(h))
            throw std::runtime_error{"DD-NeRF cameras.json declares an invalid principal point."};
        NGPDataset ds;
        for (const Json& fj : frames_json.items) {
            const std::string& file = fj.at("file_path").as_string();
            std::uint64_t hash      = 14695981039346656037ull;
            for (const unsigned char byte : std::filesystem::path{file}.filename().string()) hash = (hash ^ byte) * 1099511628211ull;
            const std::filesystem::path image = detail::frame_path(path, file, false);
            if (!std::filesystem::is_regular_file(image)) throw std::runtime_error{std::format("DD-NeRF image '{}' does not exist.", image.string())};
            NGPDataset::Frame f;
            f.rgba = detail::load_png_rgba(image, f.width, f.height);
            if (f.width != w || f.height != h)
                throw std::runtime_error{std::format("DD-NeRF image '{}' is {}x{} but cameras.json declares {}x{}.", image.string(), f.width, f.height, w, h)};
            f.camera = detail::ngp_camera(fj.at("transform_matrix"), scene_scale);
            f.focal_x = fx, f.focal_y = fy, f.principal_x = cx, f.principal_y = cy;
            (hash % 10u == 0u ? ds.test : hash % 10u == 1u ? ds.validation : ds.train).push_back(std::move(f));
        }
        if (ds.train.empty()) throw std::runtime_error{"DD-NeRF split produced no training frames."};
        if (ds.validation.empty()) throw std::runtime_error{"DD-NeRF split produced no validation frames."};
        if (ds.test.empty()) throw std::runtime_error{"DD-NeRF split produced no test frames."};
        ds.scene_scale = scene_scale;
        return ds;
    } catch (const std::exception& error) {
        return std::unexpected{std::string{error.what()}};
    }
}

}  // namespace ngp::b200::dataset
