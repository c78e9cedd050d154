// Load-time codec: nunchaku "v1 single-file" SVDQuant tensors -> the buffers
// the NVFP4 lane consumes as stored (packed e2m1 weight, cuBLAS-blocked e4m3
// block scales, row-major vectors and low-rank factors). Host code, one pass
// per tensor, no logical-domain intermediate: each stored element's
// destination is computed in closed form from the storage format.
//
// The formats are the reference's (src/gen_worker/models/svdq_layout.py):
//  * qweight I8 [N, K/2], deepcompressor's mma.sync m16n8k64 fragment
//    interleave (_FRAG / _FWD_PERM, svdq_layout.py:16-18, unpack_qweight
//    :89-110). The stored order of the nibble dimensions is
//    (n_tile, k_tile, k_pack, n_pack, n_lane, k_lane, n_pack_elem,
//    k_pack_elem, n_reg, k_reg) with k_reg = the 8 nibbles of one 32-bit word;
//    n = 128 n_tile + 16 n_pack + 8 n_pack_elem + n_lane and
//    k = 64 k_tile + 32 k_pack_elem + 8 k_lane + k_reg. A stored word holds 8
//    consecutive k of one n with even k in the low nibble of each byte, which
//    is exactly one 32-bit word of the packed e2m1 layout (pack_e2m1,
//    nvfp4_quant.py:54-56): the repack is a permutation of words.
//  * wscales E4M3 [K/16, N], pack_micro_scale's (4, 4, 8) row split
//    (_MICRO_FWD_PERM / _MICRO_ROW_DIMS, svdq_layout.py:24-25,
//    unpack_wscales :117-129). Per 128 output rows x 4 scale groups the stored
//    order is (row8, row4, row32, group4) with row = 32 row32 + 8 row4 + row8;
//    the blocked layout (to_blocked_scales, nvfp4_quant.py:72-84) puts the
//    same 512 bytes at 16 (row % 32) + 4 (row % 128 / 32) + group: a
//    permutation inside each 512-byte tile.
//  * vectors (wcscales, smooth_factor, bias): pack_scale(group_size=-1)
//    (_VEC_FWD_PERM / _VEC_ROW_DIMS, svdq_layout.py:27-28, unpack_vector
//    :132-142); per 128 elements the stored order is (a8, c4, b2, e2) for
//    i = 16 a8 + 8 b2 + 2 c4 + e2.
//  * proj_down [K, r] / proj_up [N, r] bf16: pack_lowrank_weight's 16 x 16
//    pack (_LR_* constants, svdq_layout.py:30-33, unpack_lowrank :145-162).
//    Stored order (c_pack, r_pack, n_lane8, k_lane4, n_pack2, k_pack2, k_reg2)
//    with n16 = 8 n_pack2 + n_lane8 and k16 = 8 k_pack2 + 2 k_lane4 + k_reg2;
//    down: element [16 c_pack + k16][16 r_pack + n16]; up: element
//    [16 c_pack + n16][16 r_pack + k16].
//  * quantized low-rank factors (int8 or e4m3, plain row-major, fp32 scales
//    per 32-element block along the contraction dim; dequantize_lowrank,
//    svdq_layout.py:284-306): bf16(q * scale), round to nearest even.
#include <cmath>
#include <cstdint>
#include <cstring>

namespace gwb {
namespace codec {

// qweight [N, K/2] bytes -> packed e2m1 [N, K/2] bytes. N % 128 == 0,
// K % 128 == 0 (checked by the caller).
inline void qweight_to_e2m1(const uint32_t* __restrict__ src, int64_t N, int64_t K,
                            uint32_t* __restrict__ dst) {
  const int64_t KT = K / 64;          // 64-wide k tiles
  const int64_t words_per_row = K / 8;
  const int64_t nwords = N * K / 8;
  for (int64_t s = 0; s < nwords; ++s) {
    int64_t t = s;
    const int kps = (int)(t & 1); t >>= 1;     // k_pack_elem (2)
    const int nps = (int)(t & 1); t >>= 1;     // n_pack_elem (2)
    const int kl = (int)(t & 3); t >>= 2;      // k_lane (4)
    const int nl = (int)(t & 7); t >>= 3;      // n_lane (8)
    const int np = (int)(t & 7); t >>= 3;      // n_pack (8)
    const int64_t kt = t % KT;                 // k_tile (k_pack has size 1)
    const int64_t nt = t / KT;                 // n_tile
    const int64_t n = nt * 128 + np * 16 + nps * 8 + nl;
    const int64_t kw = kt * 8 + kps * 4 + kl;  // k / 8
    dst[n * words_per_row + kw] = src[s];
  }
}

// wscales [K/16, N] e4m3 -> blocked [N/128 tiles x (K/64) tiles x 512]. N % 128
// == 0 and (K/16) % 4 == 0 (checked by the caller).
inline void wscales_to_blocked(const uint8_t* __restrict__ src, int64_t N, int64_t K,
                               uint8_t* __restrict__ dst) {
  const int64_t ncb = K / 64;                  // 4-group column tiles
  const int64_t ntiles = (N / 128) * ncb;      // stored tile order (row tile, col tile)
  for (int64_t tile = 0; tile < ntiles; ++tile) {
    const uint8_t* s = src + tile * 512;
    uint8_t* d = dst + tile * 512;             // the blocked tile order is the same
    for (int i = 0; i < 512; ++i) {
      const int e = i & 3;                     // group within the tile
      const int b = (i >> 2) & 3;              // row / 32
      const int c = (i >> 4) & 3;              // (row % 32) / 8
      const int r8 = i >> 6;                   // row % 8
      d[16 * (c * 8 + r8) + 4 * b + e] = s[i];
    }
  }
}

// pack_scale vector [n] -> row-major [n]; n % 128 == 0, elem_bytes in {1,2,4,8}.
inline void vector_unpack(const uint8_t* __restrict__ src, int64_t n, int elem_bytes,
                          uint8_t* __restrict__ dst) {
  for (int64_t s = 0; s < n; ++s) {
    int64_t t = s;
    const int e = (int)(t & 1); t >>= 1;
    const int b = (int)(t & 1); t >>= 1;
    const int c = (int)(t & 3); t >>= 2;
    const int a = (int)(t & 7); t >>= 3;
    const int64_t i = t * 128 + a * 16 + b * 8 + c * 2 + e;
    std::memcpy(dst + i * elem_bytes, src + s * elem_bytes, elem_bytes);
  }
}

// pack_lowrank_weight-packed 16-bit factor [rows, rank] -> row-major
// [rows, rank]; rows % 16 == 0, rank % 16 == 0. down: rows = in_features.
inline void lowrank_unpack(const uint16_t* __restrict__ src, int64_t rows, int64_t rank,
                           bool down, uint16_t* __restrict__ dst) {
  const int64_t RP = rank / 16;
  const int64_t total = rows * rank;
  for (int64_t s = 0; s < total; ++s) {
    int64_t t = s;
    const int rk = (int)(t & 1); t >>= 1;      // k_reg (2)
    const int kps = (int)(t & 1); t >>= 1;     // k_pack_elem (2)
    const int nps = (int)(t & 1); t >>= 1;     // n_pack_elem (2)
    const int kl = (int)(t & 3); t >>= 2;      // k_lane (4)
    const int nl = (int)(t & 7); t >>= 3;      // n_lane (8)
    const int64_t rp = t % RP;
    const int64_t cp = t / RP;
    const int n16 = nps * 8 + nl;
    const int k16 = kps * 8 + kl * 2 + rk;
    const int64_t o = down ? (cp * 16 + k16) * rank + rp * 16 + n16
                           : (cp * 16 + n16) * rank + rp * 16 + k16;
    dst[o] = src[s];
  }
}

// AWQ W4A16 qweight (TinyChat pack_w4 of deepcompressor, stored I32
// [N/4, K/2] = I16 [N/4, K]; svdq_awq.py:31-47 and its inverse pack_w4x16
// :136-147) -> packed u8 [N, K/2], even k in the low nibble. The stored 16-bit
// value t = (row group of 4, 64-code chunk, row in group, j16) holds, for
// row n = 4 group + row and u = 16 chunk + j16, the codes of k = 32 (u / 8)
// + (u % 8) + 8 i in its nibbles i = 0..3. N % 4 == 0, K % 64 == 0.
inline void awq_qweight_unpack(const uint16_t* __restrict__ src, int64_t N, int64_t K,
                               uint8_t* __restrict__ dst) {
  const int64_t chunks = K / 64;
  const int64_t total = N * K / 4;
  std::memset(dst, 0, (size_t)(N * K / 2));
  for (int64_t t = 0; t < total; ++t) {
    int64_t v = t;
    const int j16 = (int)(v & 15); v >>= 4;
    const int r4 = (int)(v & 3); v >>= 2;
    const int64_t c = v % chunks;
    const int64_t R = v / chunks;
    const int64_t n = R * 4 + r4;
    const int64_t u = c * 16 + j16;
    const uint16_t word = src[t];
    for (int i = 0; i < 4; ++i) {
      const int64_t k = 32 * (u / 8) + (u % 8) + 8 * i;
      const uint8_t code = (uint8_t)((word >> (4 * i)) & 0xF);
      dst[n * (K / 2) + k / 2] |= (k & 1) ? (uint8_t)(code << 4) : code;
    }
  }
}

inline float e4m3_to_float(uint8_t v) {
  const int e = (v >> 3) & 0xF, m = v & 7;
  float f;
  if (e == 0xF && m == 7) f = NAN;
  else if (e == 0) f = std::ldexp((float)m, -9);
  else f = std::ldexp(1.0f + (float)m / 8.0f, e - 7);
  return (v & 0x80) ? -f : f;
}

inline uint16_t float_to_bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

// q [rows, cols] (int8 or e4m3 bytes), scale fp32 blocked by 32 along
// block_dim ([rows/32, cols] or [rows, cols/32]) -> bf16 [rows, cols].
inline void lowrank_dequant(const uint8_t* __restrict__ q, const float* __restrict__ scale,
                            int64_t rows, int64_t cols, int block_dim, bool e4m3,
                            uint16_t* __restrict__ dst) {
  const int64_t scols = block_dim == 0 ? cols : cols / 32;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      const uint8_t b = q[r * cols + c];
      const float v = e4m3 ? e4m3_to_float(b) : (float)(int8_t)b;
      const float s = block_dim == 0 ? scale[(r / 32) * scols + c] : scale[r * scols + c / 32];
      dst[r * cols + c] = float_to_bf16_rne(v * s);
    }
}

}  // namespace codec
}  // namespace gwb
