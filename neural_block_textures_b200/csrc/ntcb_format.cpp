// The .ntcb container reader (layout: magic "ntcb", version 1 / 2, a header of fixed fields, per-texture channel
// counts, hidden widths, the positional spec and one record per latent level; then one section per level and one
// for the MLP, each with an 8-byte section header; bodies are LSB-first bit streams opened and closed by 6-bit
// sync markers). The field order, ranges and refusal rules follow the reference's writer and readers
// (main.cpp:2366-2630, 2762-2855); the code is this library's own.
//
// Floating-point note: the table builders below are the reference's strict-FP expressions, one IEEE operation
// at a time. This file is compiled for the x86-64 baseline (no FMA instructions), so nothing is contracted.
#include "ntcb_format.h"

#include <algorithm>
#include <cmath>
#include <cstring>

namespace ntcb {

namespace {

constexpr uint32_t kMagic = 0x6263746Eu;   // "ntcb" little-endian
constexpr int kFixedHeader = 52;
constexpr int kSyncBits = 6;
constexpr uint32_t kSyncLevel = 0x2Bu, kSyncChannel = 0x16u, kSyncMlp = 0x31u, kSyncEnd = 0x0Cu;
constexpr int kMaxUnits = 64;               // widest layer the device decode kernels take
constexpr int kEob = 64;

uint32_t sync_value(uint32_t base, int level, int channel) { return (base + 13u * (uint32_t)level + 7u * (uint32_t)channel) & 63u; }

// Little-endian fields, bounds-checked: `ok` drops on the first read past the limit.
struct Bytes {
    const uint8_t* p; size_t lim, at = 0; bool ok = true;
    Bytes(const uint8_t* p_, size_t lim_) : p(p_), lim(lim_) {}
    uint32_t u8() { if (at >= lim) { ok = false; return 0; } return p[at++]; }
    uint32_t u16() { const uint32_t a = u8(); return a | (u8() << 8); }
    uint32_t u32() { const uint32_t a = u16(); return a | (u16() << 16); }
    float f32() { const uint32_t u = u32(); float f; memcpy(&f, &u, 4); return f; }
};

// LSB-first bit stream over [begin, end) of the file.
struct Bits {
    const uint8_t* p; size_t at, end; uint64_t acc = 0; int have = 0; bool ok = true;
    Bits(const uint8_t* p_, size_t begin, size_t end_) : p(p_), at(begin), end(end_) {}
    uint32_t get(int n) {
        while (have < n) {
            if (at >= end) { ok = false; return 0; }
            acc |= (uint64_t)p[at++] << have;
            have += 8;
        }
        const uint32_t v = (uint32_t)(acc & ((1ull << n) - 1ull));
        acc >>= n; have -= n;
        return v;
    }
    void skip(uint64_t n) {   // the buffered bits first, then whole bytes without reading them, then the rest
        const int k = (int)std::min<uint64_t>(n, (uint64_t)have);
        if (k > 0) { get(k); n -= (uint64_t)k; }
        const uint64_t bytes = n / 8;
        if (at + bytes > end) { ok = false; return; }
        at += bytes;
        if (n % 8) get((int)(n % 8));
    }
    size_t next_byte() const { return at; }   // after dropping the partial byte
};

uint32_t file_hash(const uint8_t* p, size_t n) {   // FNV-1a 32, the hash field (bytes 28..31) read as zero
    uint32_t h = 2166136261u;
    for (size_t i = 0; i < n; i++) { h ^= (i >= 28 && i < 32) ? 0u : p[i]; h *= 16777619u; }
    return h;
}
bool finite32(float f) { uint32_t u; memcpy(&u, &f, 4); return (u & 0x7F800000u) != 0x7F800000u; }

int dc_field_bits(int dc_step) {   // ceil(log2(floor(512 / dc_step) + 1))
    const int levels = 512 / dc_step + 1;
    int b = 0;
    while ((1 << b) < levels) b++;
    return b;
}

bool parse_pos(const std::string& s, std::vector<int>& kinds) {
    kinds.clear();
    if (s.empty() || s == "none") return true;
    size_t a = 0;
    while (a <= s.size()) {
        size_t e = s.find(',', a);
        if (e == std::string::npos) e = s.size();
        const std::string item = s.substr(a, e - a);
        a = e + 1;
        if (item.empty()) { if (e == s.size()) break; continue; }
        if (item == "uv") kinds.push_back(0);
        else if (item == "lv1local") kinds.push_back(1);
        else return false;
        if (e == s.size()) break;
    }
    return true;
}

uint64_t weight_count(const NtcbFile& f) {
    uint64_t n = 0; int prev = f.nin;
    for (int w : f.hidden) { n += (uint64_t)w * prev + w; prev = w; }
    return n + (uint64_t)f.nout * prev + f.nout;
}

// The fewest section bytes the header's records allow (DCT levels at their floor of DC + EOB per block).
uint64_t min_section_bytes(const NtcbFile& f) {
    uint64_t total = 0;
    for (const NtcbLevelRec& L : f.lv) {
        uint64_t bits = 2 * kSyncBits;
        if (L.mode == 3) {
            const uint64_t nblk = (uint64_t)(L.W / 8) * (uint64_t)(L.H / 8);
            bits += (uint64_t)L.C * (kSyncBits + nblk * (uint64_t)(4 + dc_field_bits(L.dc_step) + 7));
        } else {
            for (int c = 0; c < L.C; c++) bits += (uint64_t)L.W * (uint64_t)L.H * (uint64_t)L.bits[c];
        }
        total += 8 + (bits + 7) / 8;
    }
    return total + 8 + (16 * weight_count(f) + 2 * kSyncBits + 7) / 8;
}

bool read_header(const uint8_t* buf, size_t n, NtcbFile& f, std::string& err) {
    if (n < 8) { err = "not an ntcb file (shorter than 8 bytes)"; return false; }
    Bytes r(buf, n);
    if (r.u32() != kMagic) { err = "not an ntcb file (bad magic)"; return false; }
    f.version = (int)r.u16();
    f.header_bytes = (int)r.u16();
    if (f.version != 1 && f.version != 2) { err = "ntcb version " + std::to_string(f.version) + " (versions 1 and 2 are read)"; return false; }
    if (f.header_bytes < kFixedHeader || (size_t)f.header_bytes > n) { err = "header length exceeds the file size (truncated or corrupt)"; return false; }
    r.lim = (size_t)f.header_bytes;
    f.img_w = (int)r.u32(); f.img_h = (int)r.u32(); f.src_w = (int)r.u32(); f.src_h = (int)r.u32();
    const uint32_t file_bytes = r.u32(), hash = r.u32();
    if (file_bytes != n) { err = "file_bytes " + std::to_string(file_bytes) + " != actual size " + std::to_string(n) + " (truncated or extended)"; return false; }
    if (file_hash(buf, n) != hash) { err = "file hash mismatch (corrupt file)"; return false; }
    f.latent_cell = (int)r.u8(); f.dct_block = (int)r.u8(); f.T = (int)r.u8(); f.nlevels = (int)r.u8();
    const int act = (int)r.u8();
    f.clamp = (int)r.u8(); f.nhidden = (int)r.u8();
    const int reserved = (int)r.u8();
    f.leak = r.f32(); f.nin = (int)r.u32(); f.nout = (int)r.u32();
    if (!r.ok) { err = "truncated header"; return false; }
    if (f.img_w < 1 || f.img_h < 1 || f.src_w < 1 || f.src_h < 1 || f.src_w > f.img_w || f.src_h > f.img_h || f.img_w > 16384 || f.img_h > 16384)
        { err = "bad image size fields"; return false; }
    if (f.T < 1 || f.T > 4 || f.nlevels < 1 || f.nlevels > 3 || act != 0 || (f.clamp != 0 && f.clamp != 1) || f.nhidden < 1 ||
        f.nhidden > 8 || reserved != 0)
        { err = "header field out of range"; return false; }
    if (!finite32(f.leak) || f.nin < 1 || f.nout < 1) { err = "bad leak, nin or nout"; return false; }
    int chan = 0;
    for (int t = 0; t < f.T; t++) {
        const int c = (int)r.u8();
        if (r.ok && c != 3) { err = "texture " + std::to_string(t) + " has " + std::to_string(c) + " channels (3 per texture are decoded)"; return false; }
        chan += c;
    }
    if (!r.ok) { err = "truncated header (channel counts)"; return false; }
    if (chan != f.nout) { err = "nout disagrees with the per-texture channel counts"; return false; }
    f.hidden.assign(f.nhidden, 0);
    for (int l = 0; l < f.nhidden; l++) {
        f.hidden[l] = (int)r.u16();
        if (r.ok && (f.hidden[l] < 1 || f.hidden[l] > 128)) { err = "bad hidden width"; return false; }
    }
    const int poslen = (int)r.u16();
    if (!r.ok || poslen >= 4096) { err = "bad positional spec length"; return false; }
    f.pos.assign((size_t)poslen, ' ');
    for (int i = 0; i < poslen; i++) f.pos[(size_t)i] = (char)r.u8();
    if (!r.ok) { err = "truncated header (positional spec)"; return false; }
    f.lv.assign((size_t)f.nlevels, NtcbLevelRec());
    int chsum = 0;
    for (int l = 0; l < f.nlevels; l++) {
        NtcbLevelRec& L = f.lv[(size_t)l];
        const std::string at = "level " + std::to_string(l) + ": ";
        L.W = (int)r.u32(); L.H = (int)r.u32(); L.C = (int)r.u16();
        const int filter = (int)r.u8();
        L.mode = (int)r.u8();
        if (!r.ok) { err = at + "truncated level record"; return false; }
        if (L.W < 1 || L.H < 1 || L.W > (1 << 20) || L.H > (1 << 20) || L.C < 1 || L.C > 128 || (filter != 0 && filter != 1) || L.mode < 0 || L.mode > 3)
            { err = at + "bad dims, filter flag or mode"; return false; }
        L.nearest = filter;
        if (l > 0 && L.mode > 1) { err = at + "qat / dct modes are only defined on level 0"; return false; }
        L.bits.assign((size_t)L.C, 0);
        for (int c = 0; c < L.C; c++) L.bits[(size_t)c] = (int)r.u8();
        if (!r.ok) { err = at + "truncated level record"; return false; }
        for (int c = 0; c < L.C; c++) {
            const int B = L.bits[(size_t)c];
            const bool ok = L.mode == 3 ? B == 0 : (L.mode == 2 ? (B >= 1 && B <= 8) : (B >= 2 && B <= 12));
            if (!ok) { err = at + "bit depth out of range for its mode"; return false; }
            if (L.mode <= 1 && B != L.bits[0]) { err = at + "per-channel depths on a grid level are not defined"; return false; }
        }
        if (L.mode == 3) {
            L.dc_step = (int)r.u8();
            const int flags = f.version >= 2 ? (int)r.u8() : 1;
            L.q.assign((size_t)L.C, 0);
            for (int c = 0; c < L.C; c++) L.q[(size_t)c] = (int)r.u8();
            if (!r.ok) { err = at + "truncated level record"; return false; }
            if (L.dc_step < 1 || L.dc_step > 64) { err = at + "dc_step out of range (1..64)"; return false; }
            if (flags & ~1) { err = at + "dct_flags has reserved bits set"; return false; }
            L.deadzone = flags & 1;
            for (int c = 0; c < L.C; c++) if (L.q[(size_t)c] < 1 || L.q[(size_t)c] > 100) { err = at + "dct quality out of range (1..100)"; return false; }
            if (f.dct_block != 8 || !L.nearest || L.W != f.img_w || L.H != f.img_h || L.W % 8 || L.H % 8 || L.C > 4)
                { err = at + "a dct level must be full-resolution, nearest, a multiple of 8 in size, with at most 4 channels"; return false; }
        } else if (l == 0 && f.dct_block != 0) { err = "dct_block must be 0 when level 0 is not DCT-coded"; return false; }
        if (L.mode == 2 && !L.nearest) { err = at + "a qat level must be nearest"; return false; }
        if (L.mode <= 1) {
            L.lo.assign((size_t)L.C, 0.0f); L.hi.assign((size_t)L.C, 0.0f);
            for (int c = 0; c < L.C; c++) { L.lo[(size_t)c] = r.f32(); L.hi[(size_t)c] = r.f32(); }
            if (!r.ok) { err = at + "truncated grid ranges"; return false; }
            for (int c = 0; c < L.C; c++)
                if (!finite32(L.lo[(size_t)c]) || !finite32(L.hi[(size_t)c]) || L.lo[(size_t)c] > L.hi[(size_t)c]) { err = at + "bad grid range"; return false; }
        }
        if (L.mode == 2) {
            L.palette.assign((size_t)L.C, std::vector<float>());
            for (int c = 0; c < L.C; c++) {
                L.palette[(size_t)c].assign((size_t)1 << L.bits[(size_t)c], 0.0f);
                for (float& v : L.palette[(size_t)c]) {
                    v = r.f32();
                    if (r.ok && !finite32(v)) { err = at + "non-finite palette value"; return false; }
                }
            }
            if (!r.ok) { err = at + "truncated palette"; return false; }
        }
        chsum += L.C;
    }
    if (r.at != (size_t)f.header_bytes) { err = "header length disagrees with its fields"; return false; }
    if (!parse_pos(f.pos, f.pos_kinds)) { err = "positional spec \"" + f.pos + "\" is not one this build reads"; return false; }
    for (int k : f.pos_kinds) if (k == 1 && f.nlevels < 2) { err = "lv1local needs a second level"; return false; }
    if (chsum + 2 * (int)f.pos_kinds.size() != f.nin) { err = "nin disagrees with the latent channels plus the positional inputs"; return false; }
    if (min_section_bytes(f) > (uint64_t)n - (uint64_t)f.header_bytes) { err = "the header's sections need more bytes than the file holds (truncated or corrupt)"; return false; }
    return true;
}

}  // namespace

float half_to_float(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    const int e = (h >> 10) & 0x1F;
    const uint32_t m = h & 0x3FFu;
    float f;
    if (e == 0) {
        f = (float)m * 5.9604644775390625e-8f;   // m * 2^-24, exact
        uint32_t u; memcpy(&u, &f, 4); u |= sign; memcpy(&f, &u, 4);
        return f;
    }
    const uint32_t u = e == 31 ? (sign | 0x7F800000u | (m << 13)) : (sign | ((uint32_t)(e - 15 + 127) << 23) | (m << 13));
    memcpy(&f, &u, 4);
    return f;
}

bool ntcb_parse(const uint8_t* buf, size_t n, NtcbFile& f, std::string& err) {
    f = NtcbFile();
    if (!read_header(buf, n, f, err)) return false;
    size_t pos = (size_t)f.header_bytes;
    auto section = [&](int kind, int level, size_t& body, size_t& len) -> bool {
        const std::string what = kind == 1 ? "level " + std::to_string(level) : std::string("the mlp");
        if (pos + 8 > n) { err = "truncated at the section header of " + what; return false; }
        Bytes r(buf + pos, 8);
        const int k = (int)r.u8(), coding = (int)r.u8(), lvl = (int)r.u8(), res = (int)r.u8();
        len = r.u32();
        if (coding != 0) { err = "section coding " + std::to_string(coding) + " (only raw fixed-width, 0, is defined)"; return false; }
        if (k != kind || lvl != level || res != 0) { err = "unexpected section header where " + what + " was expected"; return false; }
        body = pos + 8;
        if (len > n - body) { err = "section of " + what + " runs past the end of the file"; return false; }
        return true;
    };
    for (int l = 0; l < f.nlevels; l++) {
        NtcbLevelRec& L = f.lv[(size_t)l];
        const std::string at = "level " + std::to_string(l) + ": ";
        size_t body = 0, len = 0;
        if (!section(1, l, body, len)) return false;
        L.body = body; L.body_len = len;
        Bits br(buf, body, body + len);
        if (br.get(kSyncBits) != sync_value(kSyncLevel, l, 0) || !br.ok) { err = "sync marker mismatch before level " + std::to_string(l) + " body"; return false; }
        if (L.mode == 3) {
            const size_t nb = (size_t)(L.W / 8) * (size_t)(L.H / 8);
            const int dcb = dc_field_bits(L.dc_step);
            L.sym.assign(nb * (size_t)L.C * 64, 0);
            L.code.assign(nb * (size_t)L.C, 0);
            static int zz[64];
            static bool zz_ready = false;
            if (!zz_ready) { dct_zigzag(zz); zz_ready = true; }
            for (int c = 0; c < L.C; c++) {
                if (br.get(kSyncBits) != sync_value(kSyncChannel, l, c) || !br.ok) { err = "sync marker mismatch before level " + std::to_string(l) + " channel " + std::to_string(c); return false; }
                for (size_t b = 0; b < nb; b++) L.code[b * (size_t)L.C + (size_t)c] = (uint8_t)br.get(4);
                for (size_t b = 0; b < nb && br.ok; b++) {
                    int16_t* sy = L.sym.data() + (b * (size_t)L.C + (size_t)c) * 64;
                    sy[0] = (int16_t)br.get(dcb);
                    int p = 1;
                    while (p < 64 && br.ok) {
                        const int run = (int)br.get(7);
                        if (!br.ok || run == kEob) break;
                        if (run > 62) { err = at + "bad run symbol at block " + std::to_string(b); return false; }
                        p += run;
                        if (p >= 64) { err = at + "token stream runs past the 63 AC positions at block " + std::to_string(b); return false; }
                        const int mag = (int)br.get(8) + 1, sign = (int)br.get(1);
                        sy[zz[p]] = (int16_t)(sign ? -mag : mag);
                        p++;
                    }
                }
            }
            if (!br.ok) { err = at + "truncated token stream"; return false; }
        } else {
            uint64_t bitpos = kSyncBits;
            L.chan_bit.assign((size_t)L.C, 0);
            for (int c = 0; c < L.C; c++) { L.chan_bit[(size_t)c] = bitpos; bitpos += (uint64_t)L.W * L.H * (uint64_t)L.bits[(size_t)c]; }
            L.index_bit0 = kSyncBits;
            br.skip(bitpos - kSyncBits);
            if (!br.ok) { err = at + "truncated grid indices"; return false; }
        }
        if (br.get(kSyncBits) != sync_value(kSyncEnd, l, 0) || !br.ok) { err = "sync marker mismatch after level " + std::to_string(l) + " body"; return false; }
        if (br.next_byte() != body + len) { err = at + "section length disagrees with its content"; return false; }
        pos = body + len;
    }
    {
        size_t body = 0, len = 0;
        if (!section(2, 0, body, len)) return false;
        const uint64_t np = weight_count(f);
        if (len != (np * 16 + 2 * kSyncBits + 7) / 8) { err = "mlp section length disagrees with the weight count"; return false; }
        Bits br(buf, body, body + len);
        if (br.get(kSyncBits) != sync_value(kSyncMlp, f.nlevels, 0) || !br.ok) { err = "sync marker mismatch before the mlp body"; return false; }
        f.weights.assign((size_t)np, 0.0f);
        for (size_t i = 0; i < (size_t)np; i++) {
            const uint16_t h = (uint16_t)br.get(16);
            if (br.ok && (h & 0x7C00u) == 0x7C00u) { err = "non-finite mlp weight " + std::to_string(i); return false; }
            f.weights[i] = half_to_float(h);
        }
        if (!br.ok) { err = "truncated mlp section"; return false; }
        if (br.get(kSyncBits) != sync_value(kSyncEnd, f.nlevels, 0) || !br.ok) { err = "sync marker mismatch after the mlp body"; return false; }
        if (br.next_byte() != body + len) { err = "mlp section length disagrees with its content"; return false; }
        pos = body + len;
    }
    if (pos != n) { err = "trailing bytes after the mlp section"; return false; }
    int widest = f.nin;
    for (int w : f.hidden) widest = std::max(widest, w);
    if (widest > kMaxUnits) { err = "the device decoder takes at most 64 units per layer"; return false; }
    return true;
}

// ---- DCT tables
void dct_basis(float* basis) {
    const double pi = 3.14159265358979323846;
    for (int u = 0; u < 8; u++) {
        const double a = u == 0 ? std::sqrt(1.0 / 8.0) : std::sqrt(2.0 / 8.0);
        for (int x = 0; x < 8; x++) basis[u * 8 + x] = (float)(a * std::cos(pi * (2 * x + 1) * u / 16.0));
    }
}

void dct_zigzag(int* zz) {
    int k = 0;
    for (int s = 0; s < 15; s++) {
        const int x0 = s < 8 ? 0 : s - 7, x1 = s < 8 ? s : 7;
        if (s & 1) for (int x = x1; x >= x0; x--) zz[k++] = x + (s - x) * 8;
        else for (int x = x0; x <= x1; x++) zz[k++] = x + (s - x) * 8;
    }
}

namespace {
const int kJpegLuma[8][8] = {
    {4, 11, 10, 16, 24, 40, 51, 61},      {12, 12, 14, 19, 26, 58, 60, 55},   {14, 13, 16, 24, 40, 57, 69, 56},
    {14, 17, 22, 29, 51, 87, 80, 62},     {18, 22, 37, 56, 68, 109, 103, 77}, {24, 35, 55, 64, 81, 104, 113, 92},
    {49, 64, 78, 87, 103, 121, 120, 101}, {72, 92, 95, 98, 112, 100, 103, 99}};
float quality_scale(int q) {
    q = std::max(1, std::min(100, q));
    float S = q < 50 ? 5000.0f / (float)q : 200.0f - 2.0f * (float)q;
    return S * (1.0f / 100.0f);
}
float code_scale(int k) { return (float)(1.0 / ((14.0 / 64.0) * std::pow(2.0, 0.6 * k))); }
}  // namespace

void dct_steps(int q, int dc_step, int* out) {
    for (int k = 0; k < 16; k++) {
        const float ls = quality_scale(q) * code_scale(k);
        int* o = out + k * 64;
        for (int u = 0; u < 8; u++)
            for (int v = 0; v < 8; v++) {
                if (u == 0 && v == 0) { o[0] = dc_step; continue; }
                if (q >= 100) { o[u * 8 + v] = 1; continue; }
                const float i = std::min((float)v, 7.0f), j = std::min((float)u, 7.0f);
                const int i0 = (int)i, j0 = (int)j, i1 = std::min(i0 + 1, 7), j1 = std::min(j0 + 1, 7);
                const float ti = i - (float)i0, tj = j - (float)j0;
                const float a = (1.0f - ti) * (float)kJpegLuma[j0][i0] + ti * (float)kJpegLuma[j0][i1];
                const float b = (1.0f - ti) * (float)kJpegLuma[j1][i0] + ti * (float)kJpegLuma[j1][i1];
                const float base = (1.0f - tj) * a + tj * b;
                float sf = base * ls + 0.5f;
                if (!(sf >= 1.0f)) sf = 1.0f;
                if (sf > 1048576.0f) sf = 1048576.0f;
                o[u * 8 + v] = std::max(1, (int)sf);
            }
    }
}

}  // namespace ntcb
