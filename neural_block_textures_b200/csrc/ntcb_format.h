// Reader of the .ntcb bit-packed container that the reference trainer writes with --write-ntcb (version 1 and 2
// of the layout; the writer is ntcb_write, main.cpp:2637-2760, its other readers ntcb_restore, main.cpp:2762-2855,
// and load_ntcb in ntc_decode.cpp). Host code: it validates every field, locates every section, parses the DCT
// token stream and the fp16 weights; the fixed-width grid indices stay packed and are unpacked on the device.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace ntcb {

struct NtcbLevelRec {
    int W = 0, H = 0, C = 0, nearest = 0, mode = 0;   // mode 0 post-hoc grid, 1 --qes grid, 2 --qat palette, 3 DCT
    std::vector<int> bits;                            // per channel (0 for mode 3)
    std::vector<float> lo, hi;                        // modes 0 / 1
    std::vector<std::vector<float>> palette;          // mode 2: 2^bits[c] values per channel
    int dc_step = 0, deadzone = 1;                    // mode 3
    std::vector<int> q;                               // mode 3: quality per channel
    // payload
    size_t body = 0, body_len = 0;                    // byte offset / length of the section body in the file
    uint64_t index_bit0 = 0;                          // modes 0..2: bit offset of channel 0's first index inside the body
    std::vector<uint64_t> chan_bit;                   // modes 0..2: per channel, the bit offset of its first index in the body
    std::vector<int16_t> sym;                         // mode 3: [block][channel][64] symbols (natural order)
    std::vector<uint8_t> code;                        // mode 3: [block][channel] scale codes
};

struct NtcbFile {
    int version = 0, header_bytes = 0, img_w = 0, img_h = 0, src_w = 0, src_h = 0;
    int latent_cell = 0, dct_block = 0, T = 1, nlevels = 0, clamp = 0, nhidden = 0;
    float leak = 0.0f;
    int nin = 0, nout = 0;
    std::vector<int> hidden;
    std::string pos;                                  // the positional spec text
    std::vector<int> pos_kinds;                       // 0 = uv, 1 = lv1local
    std::vector<NtcbLevelRec> lv;
    std::vector<float> weights;                       // the fp16 weights as floats, the reference's flat order
};

// Parses and validates a whole container. False with a message naming the first problem.
bool ntcb_parse(const uint8_t* buf, size_t n, NtcbFile& f, std::string& err);

// IEEE binary16 -> binary32 (every half value is exact in float).
float half_to_float(uint16_t h);

// The DCT tables the reconstruction needs, from their definitions: the 8x8 basis (row u: alpha(u) cos(pi (2x + 1)
// u / 16)), the zigzag order, and the 16 step tables of one channel at quality q (dct_build_steps, main.cpp:747-781).
void dct_basis(float* basis /* 64 */);
void dct_zigzag(int* zz /* 64 */);
void dct_steps(int q, int dc_step, int* out /* 16 * 64 */);

}  // namespace ntcb
