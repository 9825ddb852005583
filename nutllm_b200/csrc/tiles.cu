/* Host packing between the reference storage and fragment tiles. */
#include <cstring>

#include "tiles.h"

namespace nut {
namespace {

inline int qget(const TileShape &s, const uint8_t *data, int64_t r, int64_t k) {
    if (r >= s.rows || k >= s.cols)
        return 0;
    const int64_t i = r * s.cols + k;
    if (s.type == 0)
        return int(int8_t(data[i]));
    const unsigned n = (i & 1) ? (data[i >> 1] >> 4) : (data[i >> 1] & 0xfu);
    return n >= 8 ? int(n) - 16 : int(n);
}

inline void qset(const TileShape &s, uint8_t *data, int64_t r, int64_t k, int q) {
    if (r >= s.rows || k >= s.cols)
        return;
    const int64_t i = r * s.cols + k;
    if (s.type == 0) {
        data[i] = uint8_t(q & 0xff);
        return;
    }
    uint8_t &b = data[i >> 1];
    b = (i & 1) ? uint8_t((b & 0x0f) | ((q & 0xf) << 4))
                : uint8_t((b & 0xf0) | (q & 0xf));
}

/* (lane, slot) -> (row offset, column offset) of the INT8 byte slot j in
 * [0, 16) of a lane's fragment. */
inline void int8_slot(int lane, int j, int &dr, int &dk) {
    const int g = lane >> 2, c = lane & 3;
    const int reg = j >> 2, e = j & 3;
    dr = g + ((reg & 1) ? 8 : 0);
    dk = 4 * c + e + ((reg & 2) ? 16 : 0);
}

} // namespace

void pack_tiles(const TileShape &s, const uint8_t *data, const uint16_t *scales,
                uint8_t *tile_data, uint16_t *tile_scales) {
    const size_t tb = s.tile_bytes();
    const int64_t src_blocks = s.cols / 32;
    for (int64_t rt = 0; rt < s.row_tiles; rt++)
        for (int64_t b = 0; b < s.blocks; b++) {
            const size_t t = s.tile_index(rt, b);
            uint8_t *out = tile_data + t * tb;
            const int64_t r0 = rt * 16, k0 = b * 32;
            for (int lane = 0; lane < 32; lane++) {
                const int g = lane >> 2, c = lane & 3;
                if (s.type == 0) {
                    for (int j = 0; j < 16; j++) {
                        int dr, dk;
                        int8_slot(lane, j, dr, dk);
                        out[16 * lane + j] = uint8_t(qget(s, data, r0 + dr, k0 + dk) & 0xff);
                    }
                } else {
                    for (int j = 0; j < 4; j++) {
                        const int lo0 = qget(s, data, r0 + g, k0 + 4 * c + j);
                        const int hi0 = qget(s, data, r0 + g + 8, k0 + 4 * c + j);
                        const int lo1 = qget(s, data, r0 + g, k0 + 16 + 4 * c + j);
                        const int hi1 = qget(s, data, r0 + g + 8, k0 + 16 + 4 * c + j);
                        out[8 * lane + j] = uint8_t((lo0 & 0xf) | ((hi0 & 0xf) << 4));
                        out[8 * lane + 4 + j] = uint8_t((lo1 & 0xf) | ((hi1 & 0xf) << 4));
                    }
                }
            }
            for (int i = 0; i < 16; i++) {
                const int64_t r = r0 + i;
                tile_scales[t * 16 + size_t(i)] =
                    (r < s.rows && b < src_blocks) ? scales[r * src_blocks + b] : 0;
            }
        }
}

void unpack_tiles(const TileShape &s, const uint8_t *tile_data,
                  const uint16_t *tile_scales, uint8_t *data, uint16_t *scales) {
    const size_t tb = s.tile_bytes();
    const int64_t src_blocks = s.cols / 32;
    if (s.type == 1)
        std::memset(data, 0, size_t((s.rows * s.cols + 1) / 2));
    for (int64_t rt = 0; rt < s.row_tiles; rt++)
        for (int64_t b = 0; b < s.blocks; b++) {
            const size_t t = s.tile_index(rt, b);
            const uint8_t *in = tile_data + t * tb;
            const int64_t r0 = rt * 16, k0 = b * 32;
            for (int lane = 0; lane < 32; lane++) {
                const int g = lane >> 2, c = lane & 3;
                if (s.type == 0) {
                    for (int j = 0; j < 16; j++) {
                        int dr, dk;
                        int8_slot(lane, j, dr, dk);
                        qset(s, data, r0 + dr, k0 + dk, int(int8_t(in[16 * lane + j])));
                    }
                } else {
                    for (int j = 0; j < 4; j++) {
                        const uint8_t w0 = in[8 * lane + j], w1 = in[8 * lane + 4 + j];
                        auto sx = [](int n) { return n >= 8 ? n - 16 : n; };
                        qset(s, data, r0 + g, k0 + 4 * c + j, sx(w0 & 0xf));
                        qset(s, data, r0 + g + 8, k0 + 4 * c + j, sx(w0 >> 4));
                        qset(s, data, r0 + g, k0 + 16 + 4 * c + j, sx(w1 & 0xf));
                        qset(s, data, r0 + g + 8, k0 + 16 + 4 * c + j, sx(w1 >> 4));
                    }
                }
            }
            for (int i = 0; i < 16; i++) {
                const int64_t r = r0 + i;
                if (r < s.rows && b < src_blocks)
                    scales[r * src_blocks + b] = tile_scales[t * 16 + size_t(i)];
            }
        }
}

} // namespace nut
