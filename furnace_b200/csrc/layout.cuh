// Device layout of quantized weights ("chunked rows") shared by host and
// device code.
//
// A weight [rows, cols] is stored row after row; every row holds exactly the
// GGUF bytes of that row (no expansion), regrouped so that a tile -- one row
// restricted to one K-chunk -- is a single contiguous, 16-byte aligned byte
// range that one bulk copy can move into shared memory:
//
//   unit   = 64 consecutive elements of K (4 Q4_K/Q6_K units per super-block,
//            2 Q8_0/Q5_0 blocks per unit); the row has U = cols/64 units.
//   chunk  = a run of <= 32 units; nch = ceil(U/32) chunks split the row as
//            evenly as whole super-blocks (K-quants) or units allow.
//   bytes  of one chunk of nu units / nsb super-blocks:
//     Q4_K  [nsb x 144 native super-blocks]
//     Q6_K  [nsb x 208 bodies][nsb x f16 d, padded to 16]
//           body = [4 x 32 nibble bytes][4 x 16 high-bit bytes][4 x 4 scales]
//           regrouped per unit of 64 consecutive elements: nibble byte i of
//           unit k holds elements 64k+i (low) and 64k+32+i (high); high-bit
//           byte i holds bits 4-5 of elements 64k+i, +16, +32, +48 (two bits
//           each, low to high); scale byte s belongs to elements 64k+16s..+16
//     Q8_0  [nu x 64 int8 quants][nu x 2 x f16 d, padded to 16]
//     Q5_0  [nu x 32 nibble bytes][nu x 2 x u32 high bits, padded][nu x 2 x f16 d, padded]
//   row stride = sum of chunk bytes (a multiple of 16).
//
// Chunks are stored plane by plane: plane c holds chunk c of every row, row
// after row, at byte offset rows * chunk_off(c); row r's chunk c (a "tile")
// starts at rows * chunk_off(c) + r * chunk_bytes(c).  Consecutive rows of one
// chunk are therefore contiguous, and a GEMV stage (16 rows x one chunk) is a
// single bulk copy.  The matrix takes rows * row_stride bytes.
//
// The same grouping decides which 16-element runs of the activation vector a
// unit multiplies (x_chunk_of below).
#pragma once

#include <cstdint>

#include "../../include/furnace.h"

#if defined(__CUDACC__)
#define FZ_HD __host__ __device__ __forceinline__
#else
#define FZ_HD inline
#endif

namespace fz {

FZ_HD uint32_t lay_units(uint32_t cols) { return (cols + 63) / 64; }  // last unit may be half (one 32-block)
FZ_HD uint32_t lay_nch(uint32_t cols) { return (lay_units(cols) + 31) / 32; }
FZ_HD bool lay_kquant(uint32_t dt) { return dt == FZ_Q4_K || dt == FZ_Q6_K; }
FZ_HD uint32_t round16u(uint32_t v) { return (v + 15u) & ~15u; }

// First unit of chunk c (c = nch gives U).
FZ_HD uint32_t lay_cu0(uint32_t dt, uint32_t cols, uint32_t c) {
  uint32_t U = lay_units(cols), nch = lay_nch(cols);
  if (c >= nch) return U;
  if (lay_kquant(dt)) {
    uint32_t nsb = U / 4;
    return 4 * (uint32_t)(((uint64_t)c * nsb) / nch);
  }
  return (uint32_t)(((uint64_t)c * U) / nch);
}

// Bytes of a chunk holding nu units.
FZ_HD uint32_t lay_chunk_bytes(uint32_t dt, uint32_t nu) {
  switch (dt) {
    case FZ_Q4_K: return 36 * nu;
    case FZ_Q6_K: return 52 * nu + round16u(nu / 2);
    case FZ_Q8_0: return 64 * nu + round16u(4 * nu);
    case FZ_Q5_0: return 32 * nu + round16u(8 * nu) + round16u(4 * nu);
    default: return 0;
  }
}

// Byte offset of chunk c inside a row.
FZ_HD uint32_t lay_chunk_off(uint32_t dt, uint32_t cols, uint32_t c) {
  uint32_t off = 0;
  for (uint32_t k = 0; k < c; k++) off += lay_chunk_bytes(dt, lay_cu0(dt, cols, k + 1) - lay_cu0(dt, cols, k));
  return off;
}

FZ_HD uint32_t lay_row_stride(uint32_t dt, uint32_t cols) { return lay_chunk_off(dt, cols, lay_nch(cols)); }

FZ_HD uint32_t lay_max_chunk_bytes(uint32_t dt, uint32_t cols) {
  uint32_t m = 0, nch = lay_nch(cols);
  for (uint32_t c = 0; c < nch; c++) {
    uint32_t b = lay_chunk_bytes(dt, lay_cu0(dt, cols, c + 1) - lay_cu0(dt, cols, c));
    m = b > m ? b : m;
  }
  return m;
}

// Byte offset of row r's tile of chunk c in a matrix of `rows` rows.
FZ_HD uint64_t lay_tile_off(uint32_t dt, uint32_t cols, uint32_t rows, uint32_t r, uint32_t c) {
  uint32_t tb = lay_chunk_bytes(dt, lay_cu0(dt, cols, c + 1) - lay_cu0(dt, cols, c));
  return (uint64_t)rows * lay_chunk_off(dt, cols, c) + (uint64_t)r * tb;
}

// Which chunk a unit belongs to.
FZ_HD uint32_t lay_chunk_of(uint32_t dt, uint32_t cols, uint32_t u) {
  uint32_t c = 0, nch = lay_nch(cols);
  while (c + 1 < nch && lay_cu0(dt, cols, c + 1) <= u) c++;
  return c;
}

// Unit u of every format covers elements 64u .. 64u+63, i.e. the 16-element
// activation runs 4u .. 4u+3.

}  // namespace fz
