/* exl3b200_layout.c -- the canonical codes plane <-> the tile-stream record the kernels stream.
 *
 * The record is exllamav3's trellis tensor for a rectangle (common/exl3_layout.h:1-17): int16
 * [cols/16][rows/16][16K], tile (tk, tn) at (tk * rows/16 + tn) * 16K, each tile the MSB-first bit stream
 * of its 256 K-bit symbols in trellis-position order; position p holds the symbol the canonical plane
 * keeps at element (n = 16 tn + c, k = 16 tk + r), (r, c) the tile place of p (common/exl3_decode.c:71-76).
 * A stacked gate_up is two records, gate rows then up rows.
 *
 * This is the loader-time relayout: a tile's 16 plane rows are read once and its 256 symbols streamed
 * through a 64-bit accumulator, both directions. Checked against the oracle's bit-by-bit transcription. */
#include "exl3b200.h"

#include <string.h>

/* (r, c) of each trellis position, and its inverse. */
static void tile_maps(int pr[256], int pc[256]) {
    static const int roff[4] = { 0, 1, 8, 9 };
    for (int p = 0; p < 256; ++p) {
        const int L = p >> 3, j = p & 7;
        pr[p] = 2 * (L & 3) + roff[j & 3];
        pc[p] = (L >> 2) + 8 * (j >> 2);
    }
}

int exl3b200_codes_to_record(const uint8_t* codes, int64_t row_bytes, int64_t rows, int64_t cols, int bits,
                             uint16_t* record) {
    int pr[256], pc[256];
    if (!codes || !record || bits < 1 || bits > 8 || rows < 0 || cols < 0 || rows % 16 || cols % 16) return -1;
    if (row_bytes < (cols * bits + 7) / 8) return -1;
    tile_maps(pr, pc);
    const int64_t nt = rows / 16, kt = cols / 16;
    const uint32_t mask = (1u << bits) - 1u;
    const int seg = 2 * bits;                        /* a row's 16 symbols of one tile: 2K whole bytes */
    for (int64_t tk = 0; tk < kt; ++tk)
        for (int64_t tn = 0; tn < nt; ++tn) {
            uint8_t sym[16][16];                     /* [c][r] */
            for (int c = 0; c < 16; ++c) {
                uint8_t b[20] = { 0 };
                memcpy(b, codes + (tn * 16 + c) * row_bytes + tk * seg, (size_t)seg);
                for (int r = 0; r < 16; ++r) {
                    const int o = r * bits;
                    sym[c][r] = (uint8_t)((((uint32_t)b[o >> 3] | ((uint32_t)b[(o >> 3) + 1] << 8)) >> (o & 7)) & mask);
                }
            }
            uint16_t* t = record + (tk * nt + tn) * 16 * bits;
            uint64_t acc = 0;
            int nb = 0, w = 0;
            for (int p = 0; p < 256; ++p) {
                acc = (acc << bits) | sym[pc[p]][pr[p]];
                nb += bits;
                if (nb >= 32) {
                    nb -= 32;
                    const uint32_t word = (uint32_t)(acc >> nb);
                    t[2 * w] = (uint16_t)(word & 0xFFFFu);
                    t[2 * w + 1] = (uint16_t)(word >> 16);
                    ++w;
                    acc &= (nb ? ((1ull << nb) - 1ull) : 0ull);
                }
            }
        }
    return 0;
}

int exl3b200_record_to_codes(const uint16_t* record, int64_t rows, int64_t cols, int bits, uint8_t* codes,
                             int64_t row_bytes) {
    int pr[256], pc[256];
    if (!codes || !record || bits < 1 || bits > 8 || rows < 0 || cols < 0 || rows % 16 || cols % 16) return -1;
    if (row_bytes < (cols * bits + 7) / 8) return -1;
    tile_maps(pr, pc);
    const int64_t nt = rows / 16, kt = cols / 16;
    const uint32_t mask = (1u << bits) - 1u;
    const int seg = 2 * bits;
    for (int64_t tk = 0; tk < kt; ++tk)
        for (int64_t tn = 0; tn < nt; ++tn) {
            uint8_t sym[16][16];
            const uint16_t* t = record + (tk * nt + tn) * 16 * bits;
            uint64_t acc = 0;
            int nb = 0, w = 0;
            for (int p = 0; p < 256; ++p) {
                if (nb < bits) {
                    const uint32_t word = (uint32_t)t[2 * w] | ((uint32_t)t[2 * w + 1] << 16);
                    ++w;
                    acc = (acc << 32) | word;
                    nb += 32;
                }
                nb -= bits;
                sym[pc[p]][pr[p]] = (uint8_t)((acc >> nb) & mask);
                acc &= (nb ? ((1ull << nb) - 1ull) : 0ull);
            }
            for (int c = 0; c < 16; ++c) {
                uint8_t b[20] = { 0 };
                for (int r = 0; r < 16; ++r) {
                    const int o = r * bits;
                    const uint32_t v = (uint32_t)sym[c][r] << (o & 7);
                    b[o >> 3] |= (uint8_t)(v & 0xFFu);
                    b[(o >> 3) + 1] |= (uint8_t)(v >> 8);
                }
                memcpy(codes + (tn * 16 + c) * row_bytes + tk * seg, b, (size_t)seg);
            }
        }
    return 0;
}
