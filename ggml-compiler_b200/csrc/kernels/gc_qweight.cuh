// Device layout of a quantized (Q4_0 / Q8_0) weight, repacked from the GGUF blocks at load.
//
// Rows are grouped in tiles of QTR = 8 rows; each row's blocks are cut into segments of QSEG = 128
// blocks (4096 values; the last segment may be shorter). A tile is stored segment after segment,
// and each (tile, segment) piece holds the 8 rows' codes block after block, then their fp16 scales:
//
//   piece(t, g) = [ codes: 8 rows x sb blocks x CB bytes ][ scales: 8 rows x sb x 2 bytes ]
//
// with CB = 16 (Q4_0, the GGUF nibble order) or 32 (Q8_0) and sb = min(QSEG, nb - g*QSEG). Every
// piece is one contiguous, 16-byte aligned range, so a GEMV streams a tile segment with a single
// bulk copy and finds every block of a row at a 16-byte boundary. Rows past the last tile's end
// are zero padding.
#pragma once

#include <cstdint>

namespace gcb {

constexpr int QTR = 8;
constexpr int QSEG = 128;

struct QW {
    const char *base;
    int64_t nb;  // blocks per row
    int cb;      // code bytes per block
};

__host__ __device__ __forceinline__ int64_t qw_tile_bytes(int64_t nb, int cb) { return (int64_t)QTR * nb * (cb + 2); }
__host__ __device__ __forceinline__ int64_t qw_seg_blocks(int64_t nb, int64_t g) {
    const int64_t r = nb - g * QSEG;
    return r < QSEG ? r : QSEG;
}
__host__ __device__ __forceinline__ int64_t qw_nseg(int64_t nb) { return (nb + QSEG - 1) / QSEG; }
__host__ __device__ __forceinline__ int64_t qw_piece_off(int64_t nb, int cb, int64_t tile, int64_t g) {
    return tile * qw_tile_bytes(nb, cb) + (int64_t)QTR * g * QSEG * (cb + 2);
}
__host__ __device__ __forceinline__ int64_t qw_piece_bytes(int64_t nb, int cb, int64_t g) {
    return (int64_t)QTR * qw_seg_blocks(nb, g) * (cb + 2);
}
__host__ __forceinline__ int64_t qw_total_bytes(int64_t rows, int64_t nb, int cb) {
    return (rows + QTR - 1) / QTR * qw_tile_bytes(nb, cb);
}

__device__ __forceinline__ const char *qw_code(const QW &w, int64_t row, int64_t blk) {
    const int64_t g = blk / QSEG, sb = qw_seg_blocks(w.nb, g);
    return w.base + qw_piece_off(w.nb, w.cb, row / QTR, g) + ((row % QTR) * sb + blk % QSEG) * w.cb;
}

__device__ __forceinline__ uint16_t qw_scale(const QW &w, int64_t row, int64_t blk) {
    const int64_t g = blk / QSEG, sb = qw_seg_blocks(w.nb, g);
    const char *p = w.base + qw_piece_off(w.nb, w.cb, row / QTR, g) + QTR * sb * w.cb;
    return ((const uint16_t *)p)[(row % QTR) * sb + blk % QSEG];
}

}  // namespace gcb
