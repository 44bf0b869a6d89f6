// tiles.cuh -- device layout of quantized matrices ("row-interleaved tiles").
//
// A matrix of N rows x K columns (K a multiple of 256) in block format f is
// stored as row groups of 32 rows.  For row group g and super-block s (256
// columns) the 32 rows' bytes form one contiguous tile:
//
//   main[g][s][c][lane]  16-byte chunk c of row 32g+lane   (C chunks per row)
//   aux [g][s][lane]     one 4-byte word per row            (Q2_K only)
//
// so a warp whose lane i owns row 32g+i reads chunk c of all 32 rows as one
// fully coalesced 512-byte transaction, and each lane accumulates its own row.
// Per format the chunks hold the reference's block bytes, reordered only where
// that lets the inner product use 4-byte integer dot products directly:
//   Q4_K (144 B/256): c0 = d, dmin, 12 scale bytes; c1..c8 = qs[0..128)
//   Q4_0 (8 x 18 B):  c0 = the eight f16 scales; c1..c8 = qs of blocks 0..7
//   Q8_0 (8 x 34 B):  c0 = the eight f16 scales; c1..c16 = qs of blocks 0..7
//   Q2_K (84 B/256):  c0 = 16 scale bytes; c1..c4 = qs with word j holding
//                     sub-block j so that bits 2k..2k+1 of byte b are element
//                     16j+4k+b; aux = d | dmin << 16
// Rows beyond N in the last group are zero-filled (they contribute nothing).
#pragma once
#include <stdint.h>

namespace nx {

struct TileGeom {
    int chunks;     // 16-byte chunks per row per super-block
    int aux_words;  // 4-byte aux words per row per super-block
};

__host__ __device__ inline TileGeom tile_geom(int fmt) {
    switch (fmt) {
    case 12: return {9, 0};   // Q4_K
    case 2: return {9, 0};    // Q4_0
    case 8: return {17, 0};   // Q8_0
    case 10: return {5, 1};   // Q2_K
    default: return {0, 0};
    }
}

__host__ __device__ inline bool tile_supported(int fmt) { return tile_geom(fmt).chunks != 0; }

// Byte sizes of the two areas for an N x K matrix.
__host__ __device__ inline size_t tile_main_bytes(int fmt, size_t n, size_t k) {
    size_t groups = (n + 31) / 32, sb = k / 256;
    return groups * sb * (size_t)tile_geom(fmt).chunks * 512;
}
__host__ __device__ inline size_t tile_aux_bytes(int fmt, size_t n, size_t k) {
    size_t groups = (n + 31) / 32, sb = k / 256;
    return groups * sb * (size_t)tile_geom(fmt).aux_words * 128;
}

}  // namespace nx
