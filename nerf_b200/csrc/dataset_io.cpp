// dataset_io.cpp -- host-side dataset I/O in the reference's format: a Blender
// "transforms" JSON (camera_angle_x, frames[].file_path, frames[].
// transform_matrix) next to RGBA8 PNG images.  The reference's driver loads
// it with nlohmann::json and stb_image one image after another
// (benchmark.cpp:148-303); here the images are decoded by a thread pool
// straight into the caller's buffer (pinned memory, ready for
// nerf_create_context), with a self-contained PNG / zlib codec:
//   - inflate (RFC 1951: stored, fixed and dynamic Huffman blocks) with the
//     zlib wrapper (RFC 1950) and its Adler-32 check;
//   - PNG (8-bit grey, grey + alpha, RGB, RGBA, palette; filter types 0-4;
//     no interlace), chunk CRC-32 checked, converted to RGBA8;
//   - a PNG writer (RGBA8, filter 0, deflate stored blocks) used to write
//     datasets and renders.
// The camera conversion of the reference's driver (world axes (x, -z, y) ->
// (x, y, z), translation * 0.33 + 0.5, fx = W / (2 tan(angle / 2)),
// c = (size - 1) / 2) is reproduced operation for operation when asked for.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "nerf_b200.h"

namespace nbio {

// ------------------------------------------------------------ checksums
uint32_t crc32(const uint8_t* p, size_t n, uint32_t crc = 0u) {
    static uint32_t table[256];
    static const bool init = [] {
        for (uint32_t i = 0; i < 256u; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
            table[i] = c;
        }
        return true;
    }();
    (void)init;
    crc = ~crc;
    for (size_t i = 0; i < n; ++i) crc = table[(crc ^ p[i]) & 0xFFu] ^ (crc >> 8);
    return ~crc;
}
uint32_t adler32(const uint8_t* p, size_t n) {
    uint32_t a = 1u, b = 0u;
    while (n) {
        const size_t m = std::min<size_t>(n, 5552u);
        for (size_t i = 0; i < m; ++i) {
            a += p[i];
            b += a;
        }
        a %= 65521u;
        b %= 65521u;
        p += m;
        n -= m;
    }
    return (b << 16) | a;
}

// ------------------------------------------------------------- inflate
struct BitReader {
    const uint8_t* p;
    size_t n, pos = 0;  // byte position
    uint32_t bitbuf = 0, bitcnt = 0;
    bool bad = false;
    uint32_t bits(uint32_t need) {  // LSB-first
        while (bitcnt < need) {
            if (pos >= n) {
                bad = true;
                return 0u;
            }
            bitbuf |= static_cast<uint32_t>(p[pos++]) << bitcnt;
            bitcnt += 8u;
        }
        const uint32_t v = need == 32u ? bitbuf : (bitbuf & ((1u << need) - 1u));
        bitbuf = need == 32u ? 0u : bitbuf >> need;
        bitcnt -= need;
        return v;
    }
    void align() {
        bitbuf = 0u;
        bitcnt = 0u;
    }
};

// Canonical Huffman code: symbols ordered by code length, then by value;
// count[l] codes of length l.
struct Huffman {
    uint16_t count[16] = {};
    std::vector<uint16_t> symbol;
    bool build(const uint8_t* lengths, uint32_t n) {
        std::fill(count, count + 16, 0);
        for (uint32_t s = 0; s < n; ++s) ++count[lengths[s]];
        count[0] = 0;
        int left = 1;
        for (int l = 1; l < 16; ++l) {
            left = (left << 1) - count[l];
            if (left < 0) return false;  // over-subscribed
        }
        uint16_t offs[16] = {};
        for (int l = 1; l < 15; ++l) offs[l + 1] = static_cast<uint16_t>(offs[l] + count[l]);
        symbol.assign(n, 0);
        for (uint32_t s = 0; s < n; ++s)
            if (lengths[s]) symbol[offs[lengths[s]]++] = static_cast<uint16_t>(s);
        return true;
    }
    // Bit by bit: codes are read MSB-first within the LSB-first stream.
    int decode(BitReader& br) const {
        int code = 0, first = 0, index = 0;
        for (int l = 1; l < 16; ++l) {
            code |= static_cast<int>(br.bits(1));
            if (br.bad) return -1;
            const int c = count[l];
            if (code - c < first) return symbol[index + (code - first)];
            index += c;
            first = (first + c) << 1;
            code <<= 1;
        }
        return -1;
    }
};

constexpr uint16_t kLenBase[29] = {3, 4, 5, 6, 7, 8, 9, 10, 11, 13, 15, 17, 19, 23, 27, 31, 35, 43, 51, 59, 67, 83, 99, 115, 131, 163, 195, 227, 258};
constexpr uint8_t kLenExtra[29] = {0, 0, 0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 2, 2, 2, 2, 3, 3, 3, 3, 4, 4, 4, 4, 5, 5, 5, 5, 0};
constexpr uint16_t kDistBase[30] = {1, 2, 3, 4, 5, 7, 9, 13, 17, 25, 33, 49, 65, 97, 129, 193, 257, 385, 513, 769, 1025, 1537, 2049, 3073, 4097, 6145, 8193, 12289, 16385, 24577};
constexpr uint8_t kDistExtra[30] = {0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 5, 6, 6, 7, 7, 8, 8, 9, 9, 10, 10, 11, 11, 12, 12, 13, 13};

bool inflate_codes(BitReader& br, const Huffman& lit, const Huffman& dist, std::vector<uint8_t>& out, size_t limit) {
    for (;;) {
        const int s = lit.decode(br);
        if (s < 0 || out.size() > limit) return false;
        if (s < 256) {
            out.push_back(static_cast<uint8_t>(s));
        } else if (s == 256) {
            return true;
        } else {
            const int li = s - 257;
            if (li >= 29) return false;
            const uint32_t len = kLenBase[li] + br.bits(kLenExtra[li]);
            const int ds = dist.decode(br);
            if (ds < 0 || ds >= 30 || br.bad) return false;
            const uint32_t d = kDistBase[ds] + br.bits(kDistExtra[ds]);
            if (br.bad || d > out.size()) return false;
            const size_t from = out.size() - d;
            for (uint32_t k = 0; k < len; ++k) {
                const uint8_t byte = out[from + k];
                out.push_back(byte);
            }
        }
    }
}

// zlib stream -> bytes; false on any malformed input or checksum mismatch.
bool zlib_inflate(const uint8_t* p, size_t n, std::vector<uint8_t>& out, size_t expect) {
    if (n < 6u) return false;
    const uint32_t cmf = p[0], flg = p[1];
    if ((cmf & 0x0Fu) != 8u || ((cmf << 8) | flg) % 31u != 0u || (flg & 0x20u)) return false;
    out.clear();
    out.reserve(expect);
    BitReader br{p + 2, n - 6};
    uint32_t last = 0;
    Huffman fixed_lit, fixed_dist;
    {
        uint8_t l[288];
        for (int i = 0; i < 144; ++i) l[i] = 8;
        for (int i = 144; i < 256; ++i) l[i] = 9;
        for (int i = 256; i < 280; ++i) l[i] = 7;
        for (int i = 280; i < 288; ++i) l[i] = 8;
        fixed_lit.build(l, 288);
        uint8_t d[30];
        std::fill(d, d + 30, 5);
        fixed_dist.build(d, 30);
    }
    do {
        last = br.bits(1);
        const uint32_t type = br.bits(2);
        if (br.bad) return false;
        if (type == 0u) {  // stored
            br.align();
            if (br.pos + 4u > br.n) return false;
            const uint32_t len = br.p[br.pos] | (br.p[br.pos + 1] << 8);
            const uint32_t nlen = br.p[br.pos + 2] | (br.p[br.pos + 3] << 8);
            if ((len ^ 0xFFFFu) != nlen) return false;
            br.pos += 4u;
            if (br.pos + len > br.n) return false;
            out.insert(out.end(), br.p + br.pos, br.p + br.pos + len);
            br.pos += len;
        } else if (type == 1u) {
            if (!inflate_codes(br, fixed_lit, fixed_dist, out, expect)) return false;
        } else if (type == 2u) {
            const uint32_t hlit = br.bits(5) + 257u, hdist = br.bits(5) + 1u, hclen = br.bits(4) + 4u;
            if (br.bad || hlit > 286u || hdist > 30u) return false;
            static const uint8_t order[19] = {16, 17, 18, 0, 8, 7, 9, 6, 10, 5, 11, 4, 12, 3, 13, 2, 14, 1, 15};
            uint8_t cl[19] = {};
            for (uint32_t i = 0; i < hclen; ++i) cl[order[i]] = static_cast<uint8_t>(br.bits(3));
            Huffman clh;
            if (br.bad || !clh.build(cl, 19)) return false;
            uint8_t lens[320] = {};
            uint32_t i = 0;
            while (i < hlit + hdist) {
                const int s = clh.decode(br);
                if (s < 0) return false;
                if (s < 16) {
                    lens[i++] = static_cast<uint8_t>(s);
                } else {
                    uint8_t v = 0;
                    uint32_t rep = 0;
                    if (s == 16) {
                        if (i == 0u) return false;
                        v = lens[i - 1];
                        rep = 3u + br.bits(2);
                    } else if (s == 17) {
                        rep = 3u + br.bits(3);
                    } else {
                        rep = 11u + br.bits(7);
                    }
                    if (br.bad || i + rep > hlit + hdist) return false;
                    while (rep--) lens[i++] = v;
                }
            }
            Huffman lit, dist;
            if (!lit.build(lens, hlit) || !dist.build(lens + hlit, hdist)) return false;
            if (!inflate_codes(br, lit, dist, out, expect)) return false;
        } else {
            return false;
        }
        if (out.size() > expect) return false;  // more data than the image holds
    } while (!last);
    // Adler-32 of the data, big-endian, after the deflate stream.
    const size_t apos = 2u + br.pos;
    if (apos + 4u > n) return false;
    const uint32_t want = (static_cast<uint32_t>(p[apos]) << 24) | (static_cast<uint32_t>(p[apos + 1]) << 16) |
                          (static_cast<uint32_t>(p[apos + 2]) << 8) | p[apos + 3];
    return want == adler32(out.data(), out.size());
}

// ----------------------------------------------------------------- PNG
uint32_t be32(const uint8_t* p) {
    return (static_cast<uint32_t>(p[0]) << 24) | (static_cast<uint32_t>(p[1]) << 16) | (static_cast<uint32_t>(p[2]) << 8) | p[3];
}
void put_be32(std::vector<uint8_t>& v, uint32_t x) {
    v.push_back(static_cast<uint8_t>(x >> 24));
    v.push_back(static_cast<uint8_t>(x >> 16));
    v.push_back(static_cast<uint8_t>(x >> 8));
    v.push_back(static_cast<uint8_t>(x));
}
const uint8_t kPngSig[8] = {0x89, 'P', 'N', 'G', '\r', '\n', 0x1A, '\n'};

bool read_file(const std::string& path, std::vector<uint8_t>& data) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) return false;
    const std::streamoff size = f.tellg();
    if (size < 0) return false;
    data.resize(static_cast<size_t>(size));
    f.seekg(0);
    return static_cast<bool>(f.read(reinterpret_cast<char*>(data.data()), size));
}

uint8_t paeth(int a, int b, int c) {
    const int p = a + b - c, pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
    return static_cast<uint8_t>((pa <= pb && pa <= pc) ? a : (pb <= pc ? b : c));
}

// PNG file -> RGBA8 (w * h * 4 bytes into out, which must hold cap bytes).
// 0 ok, 1 I/O or format error, 2 the image does not fit cap.
int png_decode(const std::vector<uint8_t>& f, uint8_t* out, uint64_t cap, uint32_t* w_out, uint32_t* h_out) {
    if (f.size() < 8u || std::memcmp(f.data(), kPngSig, 8) != 0) return 1;
    uint32_t w = 0, h = 0, depth = 0, ctype = 0;
    std::vector<uint8_t> idat, palette, trns;
    bool have_ihdr = false, have_end = false;
    for (size_t pos = 8; pos + 12u <= f.size();) {
        const uint32_t len = be32(&f[pos]);
        if (pos + 12u + len > f.size()) return 1;
        const uint8_t* type = &f[pos + 4];
        const uint8_t* data = &f[pos + 8];
        if (crc32(type, 4u + len) != be32(&f[pos + 8 + len])) return 1;
        if (!std::memcmp(type, "IHDR", 4)) {
            if (len != 13u) return 1;
            w = be32(data);
            h = be32(data + 4);
            depth = data[8];
            ctype = data[9];
            if (data[10] != 0 || data[11] != 0 || data[12] != 0) return 1;  // deflate, adaptive filter, no interlace
            have_ihdr = true;
        } else if (!std::memcmp(type, "PLTE", 4)) {
            palette.assign(data, data + len);
        } else if (!std::memcmp(type, "tRNS", 4)) {
            trns.assign(data, data + len);
        } else if (!std::memcmp(type, "IDAT", 4)) {
            idat.insert(idat.end(), data, data + len);
        } else if (!std::memcmp(type, "IEND", 4)) {
            have_end = true;
            break;
        }
        pos += 12u + len;
    }
    if (!have_ihdr || !have_end || w == 0u || h == 0u || depth != 8u) return 1;
    uint32_t ch = 0;
    switch (ctype) {
        case 0: ch = 1; break;
        case 2: ch = 3; break;
        case 3: ch = 1; break;
        case 4: ch = 2; break;
        case 6: ch = 4; break;
        default: return 1;
    }
    if (ctype == 3u && (palette.empty() || palette.size() % 3u)) return 1;
    if (w_out) *w_out = w;
    if (h_out) *h_out = h;
    const uint64_t need = static_cast<uint64_t>(w) * h * 4u;
    if (need > cap || !out) return 2;
    const size_t stride = static_cast<size_t>(w) * ch;
    std::vector<uint8_t> raw;
    if (!zlib_inflate(idat.data(), idat.size(), raw, (stride + 1u) * h)) return 1;
    if (raw.size() != (stride + 1u) * h) return 1;
    std::vector<uint8_t> prev(stride, 0), cur(stride);
    for (uint32_t y = 0; y < h; ++y) {
        const uint8_t* line = &raw[y * (stride + 1u)];
        const uint8_t ft = line[0];
        for (size_t x = 0; x < stride; ++x) {
            const int a = x >= ch ? cur[x - ch] : 0, b = prev[x], c = x >= ch ? prev[x - ch] : 0;
            int v = line[1 + x];
            switch (ft) {
                case 0: break;
                case 1: v += a; break;
                case 2: v += b; break;
                case 3: v += (a + b) >> 1; break;
                case 4: v += paeth(a, b, c); break;
                default: return 1;
            }
            cur[x] = static_cast<uint8_t>(v);
        }
        uint8_t* o = out + static_cast<size_t>(y) * w * 4u;
        for (uint32_t x = 0; x < w; ++x) {
            uint8_t r, g, b, a = 255;
            if (ctype == 6u) {
                r = cur[4 * x]; g = cur[4 * x + 1]; b = cur[4 * x + 2]; a = cur[4 * x + 3];
            } else if (ctype == 2u) {
                r = cur[3 * x]; g = cur[3 * x + 1]; b = cur[3 * x + 2];
            } else if (ctype == 4u) {
                r = g = b = cur[2 * x]; a = cur[2 * x + 1];
            } else if (ctype == 0u) {
                r = g = b = cur[x];
            } else {
                const uint32_t idx = cur[x];
                if (3u * idx + 2u >= palette.size()) return 1;
                r = palette[3 * idx]; g = palette[3 * idx + 1]; b = palette[3 * idx + 2];
                if (idx < trns.size()) a = trns[idx];
            }
            o[4 * x] = r; o[4 * x + 1] = g; o[4 * x + 2] = b; o[4 * x + 3] = a;
        }
        std::swap(prev, cur);
    }
    return 0;
}

void put_chunk(std::vector<uint8_t>& v, const char* type, const std::vector<uint8_t>& data) {
    put_be32(v, static_cast<uint32_t>(data.size()));
    const size_t at = v.size();
    v.insert(v.end(), type, type + 4);
    v.insert(v.end(), data.begin(), data.end());
    put_be32(v, crc32(&v[at], 4u + data.size()));
}

// RGBA8 -> PNG bytes (filter 0, deflate stored blocks).
std::vector<uint8_t> png_encode(const uint8_t* rgba, uint32_t w, uint32_t h) {
    std::vector<uint8_t> raw;
    const size_t stride = static_cast<size_t>(w) * 4u;
    raw.reserve((stride + 1u) * h);
    for (uint32_t y = 0; y < h; ++y) {
        raw.push_back(0);
        raw.insert(raw.end(), rgba + y * stride, rgba + (y + 1u) * stride);
    }
    std::vector<uint8_t> z = {0x78, 0x01};
    for (size_t pos = 0; pos < raw.size() || pos == 0;) {
        const size_t len = std::min<size_t>(65535u, raw.size() - pos);
        const bool last = pos + len >= raw.size();
        z.push_back(last ? 1 : 0);
        z.push_back(static_cast<uint8_t>(len));
        z.push_back(static_cast<uint8_t>(len >> 8));
        z.push_back(static_cast<uint8_t>(~len));
        z.push_back(static_cast<uint8_t>(~len >> 8));
        z.insert(z.end(), raw.begin() + pos, raw.begin() + pos + len);
        pos += len;
        if (last) break;
    }
    put_be32(z, adler32(raw.data(), raw.size()));
    std::vector<uint8_t> out(kPngSig, kPngSig + 8);
    std::vector<uint8_t> ihdr;
    put_be32(ihdr, w);
    put_be32(ihdr, h);
    ihdr.insert(ihdr.end(), {8, 6, 0, 0, 0});
    put_chunk(out, "IHDR", ihdr);
    put_chunk(out, "IDAT", z);
    put_chunk(out, "IEND", {});
    return out;
}

// ---------------------------------------------------------------- JSON
struct JValue {
    enum Kind { Null, Bool, Num, Str, Arr, Obj } kind = Null;
    double num = 0.0;
    std::string str;
    std::vector<JValue> arr;
    std::vector<std::pair<std::string, JValue>> obj;
    const JValue* get(const char* key) const {
        for (const auto& kv : obj)
            if (kv.first == key) return &kv.second;
        return nullptr;
    }
};
struct JParser {
    const std::string& s;
    size_t i = 0;
    void ws() {
        while (i < s.size() && (s[i] == ' ' || s[i] == '\n' || s[i] == '\r' || s[i] == '\t')) ++i;
    }
    bool string(std::string& out) {
        if (i >= s.size() || s[i] != '"') return false;
        ++i;
        out.clear();
        while (i < s.size() && s[i] != '"') {
            char c = s[i++];
            if (c == '\\') {
                if (i >= s.size()) return false;
                const char e = s[i++];
                switch (e) {
                    case 'n': c = '\n'; break;
                    case 't': c = '\t'; break;
                    case 'r': c = '\r'; break;
                    case 'b': c = '\b'; break;
                    case 'f': c = '\f'; break;
                    case 'u': {  // BMP code point -> UTF-8
                        if (i + 4u > s.size()) return false;
                        const uint32_t cp = static_cast<uint32_t>(std::strtoul(s.substr(i, 4).c_str(), nullptr, 16));
                        i += 4u;
                        if (cp < 0x80u) {
                            out.push_back(static_cast<char>(cp));
                        } else if (cp < 0x800u) {
                            out.push_back(static_cast<char>(0xC0u | (cp >> 6)));
                            out.push_back(static_cast<char>(0x80u | (cp & 0x3Fu)));
                        } else {
                            out.push_back(static_cast<char>(0xE0u | (cp >> 12)));
                            out.push_back(static_cast<char>(0x80u | ((cp >> 6) & 0x3Fu)));
                            out.push_back(static_cast<char>(0x80u | (cp & 0x3Fu)));
                        }
                        continue;
                    }
                    default: c = e;
                }
            }
            out.push_back(c);
        }
        if (i >= s.size()) return false;
        ++i;
        return true;
    }
    bool value(JValue& v, int depth = 0) {
        if (depth > 64) return false;
        ws();
        if (i >= s.size()) return false;
        const char c = s[i];
        if (c == '{') {
            v.kind = JValue::Obj;
            ++i;
            ws();
            if (i < s.size() && s[i] == '}') return ++i, true;
            for (;;) {
                ws();
                std::string k;
                if (!string(k)) return false;
                ws();
                if (i >= s.size() || s[i++] != ':') return false;
                JValue x;
                if (!value(x, depth + 1)) return false;
                v.obj.emplace_back(std::move(k), std::move(x));
                ws();
                if (i < s.size() && s[i] == ',') { ++i; continue; }
                return i < s.size() && s[i++] == '}';
            }
        }
        if (c == '[') {
            v.kind = JValue::Arr;
            ++i;
            ws();
            if (i < s.size() && s[i] == ']') return ++i, true;
            for (;;) {
                JValue x;
                if (!value(x, depth + 1)) return false;
                v.arr.push_back(std::move(x));
                ws();
                if (i < s.size() && s[i] == ',') { ++i; continue; }
                return i < s.size() && s[i++] == ']';
            }
        }
        if (c == '"') {
            v.kind = JValue::Str;
            return string(v.str);
        }
        if (!s.compare(i, 4, "true")) return v.kind = JValue::Bool, v.num = 1.0, i += 4, true;
        if (!s.compare(i, 5, "false")) return v.kind = JValue::Bool, v.num = 0.0, i += 5, true;
        if (!s.compare(i, 4, "null")) return v.kind = JValue::Null, i += 4, true;
        char* end = nullptr;
        v.num = std::strtod(s.c_str() + i, &end);
        if (end == s.c_str() + i) return false;
        v.kind = JValue::Num;
        i = static_cast<size_t>(end - s.c_str());
        return true;
    }
};

// ------------------------------------------------------------ Blender set
struct Blender {
    float camera_angle_x = 0.0f;
    std::vector<std::string> files;
    std::vector<float> m;  // row-major 4x4 per frame, as in the file
};

std::filesystem::path json_file_of(const char* path) {
    std::filesystem::path p{path};
    if (p.extension() != ".json") p /= "transforms_train.json";  // a dataset directory
    return p;
}

int read_blender(const char* path, Blender& b) {
    const std::filesystem::path jp = json_file_of(path);
    std::vector<uint8_t> bytes;
    if (!read_file(jp.string(), bytes)) return 1;
    const std::string text(bytes.begin(), bytes.end());
    JParser parser{text};
    JValue root;
    if (!parser.value(root) || root.kind != JValue::Obj) return 1;
    const JValue* angle = root.get("camera_angle_x");
    const JValue* frames = root.get("frames");
    if (!angle || angle->kind != JValue::Num || !frames || frames->kind != JValue::Arr || frames->arr.empty()) return 1;
    b.camera_angle_x = static_cast<float>(angle->num);
    for (const JValue& fr : frames->arr) {
        const JValue* fp = fr.get("file_path");
        const JValue* tm = fr.get("transform_matrix");
        if (!fp || fp->kind != JValue::Str || !tm || tm->kind != JValue::Arr || tm->arr.size() != 4u) return 1;
        std::filesystem::path ip = jp.parent_path() / fp->str;
        if (!ip.has_extension()) ip.replace_extension(".png");
        b.files.push_back(ip.lexically_normal().string());
        for (const JValue& row : tm->arr) {
            if (row.kind != JValue::Arr || row.arr.size() != 4u) return 1;
            for (const JValue& x : row.arr) {
                if (x.kind != JValue::Num) return 1;
                b.m.push_back(static_cast<float>(x.num));
            }
        }
    }
    return 0;
}

// The reference driver's camera convention (benchmark.cpp:148-156, 211-286):
// world axis map W (source world x, y, z = +x, -z, +y) applied to rotation and
// translation, the camera basis unchanged, translation * 0.33 + 0.5.  The
// matrix products are summed in the same order, so the results are the same
// floats.
void reference_remap(const float* src, float* dst) {
    const float W[9] = {1.0f, 0.0f, 0.0f, 0.0f, 0.0f, 1.0f, 0.0f, -1.0f, 0.0f};
    const float I[9] = {1.0f, 0.0f, 0.0f, 0.0f, 1.0f, 0.0f, 0.0f, 0.0f, 1.0f};
    const float rot[9] = {src[0], src[1], src[2], src[4], src[5], src[6], src[8], src[9], src[10]};
    const float tr[3] = {src[3], src[7], src[11]};
    float tmp[9] = {}, r2[9] = {}, t2[3] = {};
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c)
            for (int k = 0; k < 3; ++k) tmp[r * 3 + c] += W[r * 3 + k] * rot[k * 3 + c];
    for (int r = 0; r < 3; ++r)
        for (int c = 0; c < 3; ++c)
            for (int k = 0; k < 3; ++k) r2[r * 3 + c] += tmp[r * 3 + k] * I[k * 3 + c];
    for (int r = 0; r < 3; ++r)
        for (int k = 0; k < 3; ++k) t2[r] += W[r * 3 + k] * tr[k];
    for (int r = 0; r < 3; ++r) {
        volatile float scaled = t2[r] * 0.33f;  // rounded, then biased (no contraction)
        dst[4 * r + 0] = r2[3 * r + 0];
        dst[4 * r + 1] = r2[3 * r + 1];
        dst[4 * r + 2] = r2[3 * r + 2];
        dst[4 * r + 3] = scaled + 0.5f;
    }
    dst[12] = dst[13] = dst[14] = 0.0f;
    dst[15] = 1.0f;
}

// Runs fn(i) for i in [0, n) on up to n_threads threads; false if any call failed.
template <class F>
bool parallel_for(uint32_t n, uint32_t n_threads, F fn) {
    if (n_threads == 0u) n_threads = std::max(1u, std::thread::hardware_concurrency());
    n_threads = std::min(n_threads, std::max(1u, n));
    std::atomic<uint32_t> next{0};
    std::atomic<bool> ok{true};
    auto work = [&] {
        for (uint32_t i = next++; i < n && ok.load(); i = next++)
            if (!fn(i)) ok = false;
    };
    std::vector<std::thread> pool;
    for (uint32_t t = 1; t < n_threads; ++t) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    return ok.load();
}

}  // namespace nbio

extern "C" {

NERF_API NerfStatus nerf_b200_png_read(const char* path, uint8_t* rgba8, uint64_t bytes, uint32_t* width, uint32_t* height) {
    if (!path) return NERF_STATUS_INVALID_USAGE;
    std::vector<uint8_t> f;
    if (!nbio::read_file(path, f)) return NERF_STATUS_IO_ERROR;
    const int rc = nbio::png_decode(f, rgba8, rgba8 ? bytes : 0u, width, height);
    if (rc == 1) return NERF_STATUS_IO_ERROR;
    if (rc == 2) return rgba8 ? NERF_STATUS_INVALID_USAGE : NERF_STATUS_OK;  // NULL buffer: size query
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_png_write(const char* path, const uint8_t* rgba8, uint32_t width, uint32_t height) {
    if (!path || !rgba8 || width == 0u || height == 0u) return NERF_STATUS_INVALID_USAGE;
    const std::vector<uint8_t> png = nbio::png_encode(rgba8, width, height);
    std::ofstream f(path, std::ios::binary | std::ios::trunc);
    if (!f) return NERF_STATUS_IO_ERROR;
    f.write(reinterpret_cast<const char*>(png.data()), static_cast<std::streamsize>(png.size()));
    return f.good() ? NERF_STATUS_OK : NERF_STATUS_IO_ERROR;
}

NERF_API NerfStatus nerf_b200_blender_probe(const char* path, NerfB200BlenderInfo* out) {
    if (!path || !out) return NERF_STATUS_INVALID_USAGE;
    nbio::Blender b;
    if (nbio::read_blender(path, b) != 0) return NERF_STATUS_IO_ERROR;
    std::vector<uint8_t> f;
    uint32_t w = 0, h = 0;
    if (!nbio::read_file(b.files[0], f) || nbio::png_decode(f, nullptr, 0u, &w, &h) == 1) return NERF_STATUS_IO_ERROR;
    out->image_count = static_cast<uint32_t>(b.files.size());
    out->width = w;
    out->height = h;
    out->camera_angle_x = b.camera_angle_x;
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_blender_load(const char* path, uint32_t remap, uint32_t n_threads, uint8_t* images_rgba8,
                                           uint64_t images_bytes, float* cameras_4x4, float* intrinsics4) {
    if (!path || !images_rgba8 || !cameras_4x4 || !intrinsics4) return NERF_STATUS_INVALID_USAGE;
    nbio::Blender b;
    if (nbio::read_blender(path, b) != 0) return NERF_STATUS_IO_ERROR;
    std::vector<uint8_t> f;
    uint32_t w = 0, h = 0;
    if (!nbio::read_file(b.files[0], f) || nbio::png_decode(f, nullptr, 0u, &w, &h) == 1) return NERF_STATUS_IO_ERROR;
    const uint64_t per = static_cast<uint64_t>(w) * h * 4u;
    const uint32_t n = static_cast<uint32_t>(b.files.size());
    if (images_bytes < per * n) return NERF_STATUS_INVALID_USAGE;
    std::atomic<int> status{0};  // 1 I/O, 2 size mismatch
    const bool ok = nbio::parallel_for(n, n_threads, [&](uint32_t i) {
        std::vector<uint8_t> bytes;
        uint32_t wi = 0, hi = 0;
        if (!nbio::read_file(b.files[i], bytes)) return status = 1, false;
        const int rc = nbio::png_decode(bytes, images_rgba8 + per * i, per, &wi, &hi);
        if (rc != 0 || wi != w || hi != h) return status = (rc == 1 ? 1 : 2), false;
        return true;
    });
    if (!ok) return status.load() == 2 ? NERF_STATUS_INVALID_USAGE : NERF_STATUS_IO_ERROR;
    for (uint32_t i = 0; i < n; ++i) {
        if (remap) {
            nbio::reference_remap(b.m.data() + 16u * i, cameras_4x4 + 16u * i);
        } else {
            std::memcpy(cameras_4x4 + 16u * i, b.m.data() + 16u * i, 64u);
        }
    }
    // benchmark.cpp:252-256: fx = fy = (0.5 W) / tan(angle / 2), c = 0.5 (size - 1).
    const float wf = static_cast<float>(w), hf = static_cast<float>(h);
    const float fx = 0.5f * wf / std::tan(b.camera_angle_x * 0.5f);
    intrinsics4[0] = fx;
    intrinsics4[1] = fx;
    intrinsics4[2] = 0.5f * (wf - 1.0f);
    intrinsics4[3] = 0.5f * (hf - 1.0f);
    return NERF_STATUS_OK;
}

NERF_API NerfStatus nerf_b200_blender_write(const char* dir, const uint8_t* images_rgba8, const float* cameras_4x4, uint32_t n,
                                            uint32_t width, uint32_t height, float camera_angle_x, uint32_t n_threads) {
    if (!dir || !images_rgba8 || !cameras_4x4 || n == 0u || width == 0u || height == 0u) return NERF_STATUS_INVALID_USAGE;
    std::error_code ec;
    const std::filesystem::path d{dir};
    std::filesystem::create_directories(d / "train", ec);
    if (ec) return NERF_STATUS_IO_ERROR;
    const uint64_t per = static_cast<uint64_t>(width) * height * 4u;
    const bool ok = nbio::parallel_for(n, n_threads, [&](uint32_t i) {
        char name[64];
        std::snprintf(name, sizeof(name), "r_%u.png", i);
        return nerf_b200_png_write((d / "train" / name).string().c_str(), images_rgba8 + per * i, width, height) == NERF_STATUS_OK;
    });
    if (!ok) return NERF_STATUS_IO_ERROR;
    std::ofstream f(d / "transforms_train.json", std::ios::trunc);
    if (!f) return NERF_STATUS_IO_ERROR;
    char buf[128];
    std::snprintf(buf, sizeof(buf), "{\n  \"camera_angle_x\": %.9g,\n  \"frames\": [\n", static_cast<double>(camera_angle_x));
    f << buf;
    for (uint32_t i = 0; i < n; ++i) {
        f << "    {\"file_path\": \"./train/r_" << i << "\", \"transform_matrix\": [";
        for (int r = 0; r < 4; ++r) {
            f << (r ? ", [" : "[");
            for (int c = 0; c < 4; ++c) {
                std::snprintf(buf, sizeof(buf), "%s%.9g", c ? ", " : "", static_cast<double>(cameras_4x4[16u * i + 4 * r + c]));
                f << buf;
            }
            f << "]";
        }
        f << "]}" << (i + 1u < n ? ",\n" : "\n");
    }
    f << "  ]\n}\n";
    return f.good() ? NERF_STATUS_OK : NERF_STATUS_IO_ERROR;
}

}  // extern "C"
