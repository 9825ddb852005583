#pragma once
/* Device weight layout for the tensor-pipe quantised products.
 *
 * A quantised [rows][cols] matrix (reference storage, block 32 along each
 * row, cols % 32 == 0) is stored as fragment tiles: one tile per 16 rows
 * ("row tile") x 32 columns (one quantisation block), ordered
 * [row tile][block].  A tile holds exactly the A-operand registers of one
 * mma.sync.m16n8k32 (s8) for the 32 lanes of a warp, so a lane fetches its
 * fragment with one contiguous 16-byte (INT8) or 8-byte (INT4) read:
 *
 *   lane L = 4g + c (g = L / 4, c = L % 4), rows g and g + 8 of the tile,
 *   columns 4c..4c+3 ("lo") and 16+4c..16+4c+3 ("hi").
 *   INT8 tile (512 B), lane bytes [16L, 16L+16):
 *     a0 = q[g][lo]  a1 = q[g+8][lo]  a2 = q[g][hi]  a3 = q[g+8][hi]
 *   INT4 tile (256 B), lane bytes [8L, 8L+8):
 *     word0 byte j = q[g][4c+j] | q[g+8][4c+j] << 4          (nibbles)
 *     word1 byte j = q[g][16+4c+j] | q[g+8][16+4c+j] << 4
 *     The kernel widens them with two masks to bytes 16*q (exact signed
 *     int8): a0 = (word0 << 4) & 0xF0F0F0F0, a1 = word0 & 0xF0F0F0F0, ...
 *
 * Three tile orders serve the three ways a matrix is split across CTAs:
 *   row-major    [row tile][block]            a CTA owns whole row tiles
 *   pair-column  [block / 2][row tile][2]     a CTA owns one block pair
 *                (K columns 64 P .. 64 P + 63) of a range of row tiles
 *   block-column [block][row tile]            a CTA owns whole K blocks;
 *                row tiles are padded to an even count so consecutive
 *                tiles pair up
 * In every order a CTA's share is one contiguous run of tiles.
 *
 * Scales are stored beside the data in the same tile order, 16 fp16 bits
 * per tile.
 * Rows are padded to a multiple of 16 and blocks to an even count with
 * zero weights and zero scales, which contribute exactly nothing.  The
 * packing is a byte permutation of the reference storage; unpack() inverts
 * it, and the tests check the round trip bit for bit.
 */
#include <cstddef>
#include <cstdint>
#include <vector>

namespace nut {

enum TileOrder : int { kRowMajor = 0, kPairColumn = 1, kBlockColumn = 2 };

struct TileShape {
    int64_t rows = 0, cols = 0;
    int type = 0;          /* 0 INT8, 1 INT4 */
    int64_t row_tiles = 0; /* ceil(rows / 16) (even for kBlockColumn) */
    int64_t blocks = 0;    /* ceil(cols / 32) rounded up to even */
    int order = kRowMajor;

    static TileShape of(int64_t rows, int64_t cols, int type, int order = kRowMajor) {
        TileShape s;
        s.rows = rows;
        s.cols = cols;
        s.type = type;
        s.order = order;
        s.row_tiles = (rows + 15) / 16;
        if (order == kBlockColumn)
            s.row_tiles = (s.row_tiles + 1) / 2 * 2;
        const int64_t b = (cols + 31) / 32;
        s.blocks = (b + 1) / 2 * 2;
        return s;
    }
    /* Position of tile (row tile rt, block b) in the stored sequence. */
    size_t tile_index(int64_t rt, int64_t b) const {
        if (order == kPairColumn)
            return size_t(((b >> 1) * row_tiles + rt) * 2 + (b & 1));
        if (order == kBlockColumn)
            return size_t(b * row_tiles + rt);
        return size_t(rt * blocks + b);
    }
    size_t tile_bytes() const { return type == 0 ? 512 : 256; }
    size_t tiles() const { return size_t(row_tiles * blocks); }
    size_t data_bytes() const { return tiles() * tile_bytes(); }
    size_t scale_count() const { return tiles() * 16; }
};

/* Reference storage -> fragment tiles (cols % 32 == 0 required). */
void pack_tiles(const TileShape &s, const uint8_t *data, const uint16_t *scales,
                uint8_t *tile_data, uint16_t *tile_scales);
/* Fragment tiles -> reference storage (exact inverse of pack_tiles). */
void unpack_tiles(const TileShape &s, const uint8_t *tile_data,
                  const uint16_t *tile_scales, uint8_t *data, uint16_t *scales);

} // namespace nut
