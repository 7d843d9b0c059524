// Block formats of the two expert weight types and their device decoders.
//
// ggml block layout (32 elements per block; gguf/constants.py:4251,4264):
//   IQ4_NL : fp16 d, 16 bytes of nibbles                      (18 bytes)
//   MXFP4  : e8m0 e, 16 bytes of nibbles                      (17 bytes)
// In both, byte j holds element j in its low nibble and element j + 16 in
// its high nibble. An element is scale * code[nibble]:
//   IQ4_NL : d * kvalues_iq4nl[q]   (int8 codebook, 16 entries)
//   MXFP4  : 2^(e-128) * kvalues_mxfp4[q]  (e2m1 values doubled, so that the
//            codebook is integer; 2^(e-128) is ggml's "e8m0 to fp32 half")
//
// Device pool layout (this library's, per slot, written by the fill path):
//   qs    : [K/32][N][16 B]   block-major, rows of one block contiguous
//   scale : IQ4_NL: fp16 [K/32][N];
//           MXFP4 : e8m0 bytes in 512-byte chunks, one per (4 blocks, 128
//           rows): chunk (b/4, n/128) holds row r = n%128 of block b at
//           byte (r%32)*16 + (r/32)*4 + b%4. That is the order the tensor
//           core's scale-factor copy (tcgen05.cp 32x128b, 4-way broadcast)
//           takes, so a chunk moves from the pool to tensor memory as is.
// With lane = row, a warp reading one block column loads 32 x 16 contiguous
// bytes, so every weight load in the CUDA-core matmul is a coalesced 128-bit
// load; 128 rows of one block column (2 KB) are one bulk copy for the
// tensor-core matmul.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace msb {

// Codebooks packed four int8 per word, entry i in byte i % 4 of word i / 4.
// IQ4_NL: -127 -104 -83 -65 | -49 -35 -22 -10 | 1 13 25 38 | 53 69 89 113
// MXFP4 : 0 1 2 3 | 4 6 8 12 | 0 -1 -2 -3 | -4 -6 -8 -12
struct Codebook { uint32_t w0, w1, w2, w3; };
__host__ __device__ constexpr Codebook codebook_iq4nl() {
  return {0xBFAD9881u, 0xF6EADDCFu, 0x26190D01u, 0x71594535u};
}
__host__ __device__ constexpr Codebook codebook_mxfp4() {
  return {0x03020100u, 0x0C080604u, 0xFDFEFF00u, 0xF4F8FAFCu};
}

// 2^(e-128) as f32, exact for every e (denormal below e = 2).
__device__ __forceinline__ float e8m0_half(uint32_t e) {
  return e >= 2 ? __uint_as_float((e - 1) << 23) : __uint_as_float(0x00200000u << e);
}

// Decodes one word of packed nibbles (bytes j..j+3 of a block) to eight int8
// codes in the interleaved element order used for activations:
//   lo = {x[j], x[j+16], x[j+1], x[j+17]}, hi = {x[j+2], x[j+18], x[j+3], x[j+19]}
// Each 16-entry lookup is two 8-entry byte permutes (entries 0-7 and 8-15,
// indexed by the nibble's low three bits) and a third permute that picks,
// per byte, the half named by the nibble's high bit.
__device__ __forceinline__ void decode_nibbles(uint32_t q, const Codebook &cb,
                                               uint32_t &lo, uint32_t &hi) {
  const uint32_t idx = q & 0x77777777u;
  const uint32_t pick = ((q >> 1) & 0x44444444u) | 0x32103210u;
  uint32_t a = __byte_perm(cb.w0, cb.w1, idx);
  uint32_t b = __byte_perm(cb.w2, cb.w3, idx);
  lo = __byte_perm(a, b, pick);
  const uint32_t idx_hi = idx >> 16;
  a = __byte_perm(cb.w0, cb.w1, idx_hi);
  b = __byte_perm(cb.w2, cb.w3, idx_hi);
  hi = __byte_perm(a, b, pick >> 16);
}

// Byte offset of the scale of (block b, row n) within a slot's scale region
// (N rows and nb blocks stored per slot). MXFP4: one 512-byte record per
// (128-row tile, chunk of 4 blocks), tile-major, so a tile's consecutive
// chunks are contiguous; inside a record row r of the tile is byte
// (r % 32) * 16 + (r / 32) * 4 + (b % 4) -- the tensor core's 32x4
// scale-factor atom.
__host__ __device__ __forceinline__ int64_t scale_offset(bool mx, int64_t b, int64_t n,
                                                         int64_t N, int64_t nb) {
  if (!mx) return (b * N + n) * 2;
  const int64_t r = n & 127;
  return ((n >> 7) * ((nb + 3) >> 2) + (b >> 2)) * 512 + (r & 31) * 16 + (r >> 5) * 4 + (b & 3);
}

__host__ __device__ __forceinline__ int64_t scale_region_bytes(bool mx, int64_t nb, int64_t N) {
  return mx ? ((nb + 3) / 4) * ((N + 127) / 128) * 512 : nb * N * 2;
}

// Byte position of element j (0..31) of a block in the interleaved order.
__host__ __device__ __forceinline__ int interleaved_pos(int j) {
  const int jj = j & 15;
  return 8 * (jj >> 2) + 2 * (jj & 3) + (j >> 4);
}

}  // namespace msb
