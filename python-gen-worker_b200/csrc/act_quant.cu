// Activation kernels (memory-bound, one pass over x):
//  * act_int4_kernel: smoothing divide -> bf16, per-64-group symmetric INT4
//    with fp16 scale, packed sign-magnitude nibbles (even k in the low nibble), fused with the
//    rank-r low-rank down-projection la = x·L1 on RAW x (mma.sync bf16).
//  * act_int8_kernel: per-token symmetric INT8 with fp32 scale.
// Numerics follow the reference's quantiser structure
// (src/gen_worker/models/nvfp4_quant.py:92-103): fp32 amax, scale rounded to
// its storage dtype first, IEEE divide by the rounded scale, round
// half-to-even, clamp.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include "gwb.h"
#include "ptx.cuh"

namespace gwb {

// warps per CTA (splitting K round-robin in 64-wide chunks): 16 warps of
// 128 registers fill an SM with one CTA, so a small token count (one 16-row
// tile per CTA, e.g. 132 tiles for a 2112-token shard) still runs 16 warps
// per SM; ranks above 64 keep 8 warps with the larger register budget. The
// count never depends on M, so a row's results do not depend on the shard size.
template <int NB> __host__ __device__ constexpr int act_warps() { return NB > 8 ? 8 : 16; }

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// a / b given rb = RN(1/b), correctly rounded whenever the quotient is a
// normal number (Markstein's theorem: with q0 = RN(a * rb) and the exact
// remainder r = a - b * q0 from an FMA, RN(q0 + r * rb) = RN(a / b)).
// A quotient below 2^-126 cannot change any code or scale produced here:
// group scales are at least 2^-24, so such values quantise to 0 and cannot
// be a group's amax unless every value of the group is below 2^-126, in
// which case the scale clamps to 2^-24 whatever their exact values.
__device__ __forceinline__ float div_rn(float a, float b, float rb) {
  const float q = a * rb;
  const float r = fmaf(-q, b, a);
  return fmaf(r, rb, q);
}

// sign-magnitude nibble of clamp(rint(v/s), -7, 7): bit 3 = sign, bits 0-2 = |q|.
// |q| <= 7.5 here, so min(|q|, 7) + 2^23 rounds half-to-even to the integer
// magnitude in the low mantissa bits (rint(|q|) = |rint(q)|).
__device__ __forceinline__ uint32_t q4(float v, float s, float rs) {
  const float q = div_rn(v, s, rs);
  const uint32_t mag = __float_as_uint(fminf(fabsf(q), 7.0f) + 8388608.0f) & 7u;
  return mag | ((q < 0.0f && mag != 0u) ? 8u : 0u);
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Pairwise a / b given rb = RN(1/b) (the div_rn rule on f32x2 lanes; the
// packed FMUL2 / FFMA2 round each lane exactly like their scalar forms).
__device__ __forceinline__ float2 div2_rn(float2 a, float2 b, float2 rb) {
  const float2 q = __fmul2_rn(a, rb);
  const float2 r = __ffma2_rn(make_float2(-q.x, -q.y), b, a);
  return __ffma2_rn(r, rb, q);
}

// sign-magnitude nibbles of clamp(rint(v/s), -7, 7) for a pair (see q4).
__device__ __forceinline__ uint32_t q4x2(float2 v, float2 s, float2 rs) {
  const float2 q = div2_rn(v, s, rs);
  const float2 m = __fadd2_rn(make_float2(fminf(fabsf(q.x), 7.0f), fminf(fabsf(q.y), 7.0f)),
                              make_float2(8388608.0f, 8388608.0f));
  const uint32_t m0 = __float_as_uint(m.x) & 7u, m1 = __float_as_uint(m.y) & 7u;
  return (m0 | ((q.x < 0.0f && m0 != 0u) ? 8u : 0u)) |
         ((m1 | ((q.y < 0.0f && m1 != 0u) ? 8u : 0u)) << 4);
}

// GEMM operand bytes (e4m3 of q * 2^-9: sign bit 7, magnitude in bits 0-2)
// of clamp(rint(v/s), -7, 7) for a pair. The magnitude is non-zero exactly
// when |v/s| > 0.5 (0.5 rounds to even 0), so the sign bit is set when
// v/s < -0.5: no separate test of the magnitude.
__device__ __forceinline__ void q8x2(float2 v, float2 s, float2 rs, uint32_t& b0, uint32_t& b1) {
  const float2 q = div2_rn(v, s, rs);
  const float2 m = __fadd2_rn(make_float2(fminf(fabsf(q.x), 7.0f), fminf(fabsf(q.y), 7.0f)),
                              make_float2(8388608.0f, 8388608.0f));
  b0 = (__float_as_uint(m.x) & 7u) | (q.x < -0.5f ? 0x80u : 0u);
  b1 = (__float_as_uint(m.y) & 7u) | (q.y < -0.5f ? 0x80u : 0u);
}

// Two f32 -> e4m3 bytes, round to nearest even, saturating: `hi` in bits
// 8-15, `lo` in bits 0-7.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Clear the sign of every byte whose magnitude bits are zero (a negative
// quotient that rounds to 0 converts to e4m3 -0; the operand byte is +0).
__device__ __forceinline__ uint32_t e4m3_no_neg_zero(uint32_t w) {
  const uint32_t nz = (w & 0x7F7F7F7Fu) + 0x7F7F7F7Fu;   // bit 7 set where bits 0-6 != 0
  return w & (nz | 0x7F7F7F7Fu);
}

// GEMM operand bytes of 16 elements whose quotients satisfy |v/s| <= 7.25:
// d = RN(v/s) * 2^-9 by the div_rn steps on exactly scaled operands
// (s * 2^9 and RN(1/s) * 2^-9 are exact, so every step is the unscaled step
// times 2^-9; only quotients below 2^-117 could differ, and those convert to
// 0 either way), then e4m3 RN of d = rint(v/s) * 2^-9, the subnormal code
// 0 000 |q|. Byte order as q8x2: lo = elements 0 2 4 6, hi = 1 3 5 7,
// e23 = 8 10 12 14 | 9 11 13 15.
__device__ __forceinline__ void e4m3_seg16(const float2 (&v)[8], float s, float rs,
                                           uint32_t& lo, uint32_t& hi, uint32_t* e23) {
  const float2 sp = make_float2(s * 512.0f, s * 512.0f);
  const float2 rp = make_float2(rs * 0.001953125f, rs * 0.001953125f);
  float2 d[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) d[j] = div2_rn(v[j], sp, rp);
  lo = e4m3_no_neg_zero(cvt_e4m3x2(d[1].x, d[0].x) | (cvt_e4m3x2(d[3].x, d[2].x) << 16));
  hi = e4m3_no_neg_zero(cvt_e4m3x2(d[1].y, d[0].y) | (cvt_e4m3x2(d[3].y, d[2].y) << 16));
  e23[0] = e4m3_no_neg_zero(cvt_e4m3x2(d[5].x, d[4].x) | (cvt_e4m3x2(d[7].x, d[6].x) << 16));
  e23[1] = e4m3_no_neg_zero(cvt_e4m3x2(d[5].y, d[4].y) | (cvt_e4m3x2(d[7].y, d[6].y) << 16));
}

// Quantise 16 consecutive raw elements (8 bf16x2 words) of one row-group
// segment: smoothing divide rounded to bf16, then the group's INT4 codes.
// The 4 lanes of a quad hold the 64 elements of one group. E4M3: write the
// GEMM operand form (elements 0 2 4 6 | 1 3 5 7 | 8 10 12 14 | 9 11 13 15
// as e4m3 bytes, the order unpack8_e4m3 gives) into lo, hi, e2, e3;
// otherwise the packed sign-magnitude nibbles into lo, hi.
template <bool E4M3 = false>
__device__ __forceinline__ void quant_seg16(const uint32_t (&xw)[8], const float (&sm)[16],
                                            const float (&rsm)[16], bool has_smooth,
                                            uint32_t& lo, uint32_t& hi, __half& scale_out,
                                            uint32_t* e23 = nullptr) {
  float2 v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float2 p = make_float2(bf_lo(xw[j]), bf_hi(xw[j]));
    if (has_smooth) {
      const float2 q = div2_rn(p, make_float2(sm[2 * j], sm[2 * j + 1]),
                               make_float2(rsm[2 * j], rsm[2 * j + 1]));
      const __nv_bfloat162 hb = __float22bfloat162_rn(q);
      p = __bfloat1622float2(hb);
    }
    v[j] = p;
  }
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) amax = fmaxf(amax, fmaxf(fabsf(v[j].x), fabsf(v[j].y)));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  float s32 = __fdiv_rn(amax, 7.0f);
  s32 = fminf(fmaxf(s32, 5.9604644775390625e-08f), 65504.0f);
  const __half sh = __float2half_rn(s32);
  const float s = __half2float(sh);
  const float rs = __frcp_rn(s);
  const float2 s2 = make_float2(s, s), rs2 = make_float2(rs, rs);
  lo = 0;
  hi = 0;
  if constexpr (E4M3) {
    if (amax <= 7.25f * s) {
      // |v/s| <= 7.25, so rint(v/s) needs no clamp and the e4m3 conversion
      // of (v/s) * 2^-9 (subnormal range, spacing 2^-9, round half to even)
      // is the operand byte itself
      e4m3_seg16(v, s, rs, lo, hi, e23);
      scale_out = sh;
      return;
    }
    uint32_t e2 = 0, e3 = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t b0, b1;
      q8x2(v[j], s2, rs2, b0, b1);
      lo |= b0 << (8 * j);
      hi |= b1 << (8 * j);
      q8x2(v[4 + j], s2, rs2, b0, b1);
      e2 |= b0 << (8 * j);
      e3 |= b1 << (8 * j);
    }
    e23[0] = e2;
    e23[1] = e3;
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) lo |= q4x2(v[j], s2, rs2) << (8 * j);
#pragma unroll
    for (int j = 0; j < 4; ++j) hi |= q4x2(v[4 + j], s2, rs2) << (8 * j);
  }
  scale_out = sh;
}

// One scale-operand row: the 16-bit scale `bits` at k = g mod 8, zeros at the
// other seven k (the row of group g in the one-hot [G, R, 8] form).
__device__ __forceinline__ uint4 onehot_k8(uint32_t bits, int g) {
  const uint32_t w = bits << (16 * (g & 1));
  const int q = (g >> 1) & 3;
  return make_uint4(q == 0 ? w : 0u, q == 1 ? w : 0u, q == 2 ? w : 0u, q == 3 ? w : 0u);
}

// Host helpers defined with the GEMM launches (same translation unit).
static int make_tmap(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize,
                     uint64_t cols, uint64_t rows, uint32_t bx, uint32_t by,
                     CUtensorMapSwizzle sw);
static int sm_count();

namespace actq {
// x arrives by TMA in 16-row x 64-column bf16 boxes (2 KB, 128-byte rows,
// SWIZZLE_128B), one private ring of kStages boxes per warp.
#ifndef GWB_ACT_STAGES
#define GWB_ACT_STAGES 2
#endif
constexpr int kStages = GWB_ACT_STAGES;
constexpr int kBoxBytes = 16 * 128;
template <int NB> __host__ __device__ constexpr size_t smem_bytes() {
  return 1024 + (size_t)act_warps<NB>() * kStages * kBoxBytes   // x rings
         + (size_t)act_warps<NB>() * 64 * sizeof(float)          // per-warp 1/smooth
         + (size_t)act_warps<NB>() * 16 * NB * 8 * sizeof(float)  // low-rank partials
         + (size_t)act_warps<NB>() * kStages * sizeof(uint64_t);  // ring barriers
}
}  // namespace actq

// Wait for a copy still in flight while unwinding after a failed wait:
// bounded, and not cut short by the error flag the failure already set.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  const long long start = clock64();
  const long long limit = *((volatile long long*)&gwb_wait_limit);
  while (!mbar_try_wait(bar, parity) && clock64() - start <= limit) {
  }
}

// NB = padded rank / 8 (0 = no low-rank branch). Persistent: CTA b takes the
// 16-row tiles b, b + gridDim.x, ...; within a tile its act_warps<NB>()
// warps split K round-robin in 64-wide chunks (chunk kc to warp kc % W). Each
// warp walks its (tile, chunk) items in order through a private TMA ring of
// x boxes, so the next tile's first chunks are in flight while this tile's
// low-rank partials are reduced.
// MMA_FORM = false writes the interchange form: packed codes u8 [M, K/2] and
// ascale f16 [M, K/64]. MMA_FORM = true writes the GEMM operand form: codes
// u8 [M, K] as e4m3 bytes of q * 2^-9 in the within-8 operand order
// (unpack8_e4m3), and the scales as scale-operand rows f16 [K/64, M, 8]
// (group g's scale at k = g mod 8, zeros elsewhere: one 16-byte TMA row per
// matrix row).
// la = bf16(x · L1) on raw x: each warp accumulates its K chunks with
// mma.sync; the per-warp partials are summed in a fixed order through
// shared memory, so la is deterministic and independent of M and the grid.
template <int NB, bool MMA_FORM>
__global__ void __launch_bounds__(act_warps<NB>() * 32, 1)
act_int4_kernel(const __grid_constant__ CUtensorMap tmX, const __nv_bfloat16* __restrict__ smooth,
                const __nv_bfloat16* __restrict__ down_t, uint8_t* __restrict__ codes,
                __half* __restrict__ ascale, __nv_bfloat16* __restrict__ la, int M, int K) {
  using namespace actq;
  constexpr int RP = NB * 8;
  constexpr int W = act_warps<NB>();
  constexpr int S = kStages;
  extern __shared__ uint8_t act_smem_raw[];
  uint8_t* base = act_smem_raw + ((1024u - (smem_u32(act_smem_raw) & 1023u)) & 1023u);
  uint8_t* xs = base;                                                  // [W][S][2 KB]
  float* rsw = reinterpret_cast<float*>(xs + W * S * kBoxBytes);       // [W][64]
  float* red = rsw + W * 64;                                           // [W][16][RP]
  uint64_t* bars = reinterpret_cast<uint64_t*>(red + W * 16 * RP);     // [W][S]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int nchunks = K / 64;
  const int G = K / 64;
  const int ntiles = (M + 15) / 16;
  const bool has_smooth = smooth != nullptr;
  uint8_t* my_xs = xs + warp * S * kBoxBytes;
  uint64_t* my_bar = bars + warp * S;
  float* my_rs = rsw + warp * 64;

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&my_bar[s], 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmX);
  }
  __syncwarp();

  // this warp's chunks per tile and tiles: item i = (tile i / per, chunk i % per)
  const int per = nchunks > warp ? (nchunks - warp + W - 1) / W : 0;
  const int my_tiles =
      ntiles > (int)blockIdx.x ? (ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  const int total = per * my_tiles;
  int issued = 0;
  auto issue = [&](int i) {
    if (i >= total) return;
    if (lane == 0) {
      const int tile = blockIdx.x + (i / per) * gridDim.x;
      const int kc = warp + (i % per) * W;
      const int s = i % S;
      mbar_arrive_expect_tx(&my_bar[s], kBoxBytes);
      tma_load_2d(my_xs + s * kBoxBytes, &tmX, &my_bar[s], kc * 64, tile * 16);
    }
    issued = i + 1;
  };
  for (int i = 0; i < S; ++i) issue(i);

  bool ok = true;
  int item = 0, failed_at = -1;   // first item whose wait ran out
  for (int t = 0; t < my_tiles; ++t) {
    const int tile = blockIdx.x + t * gridDim.x;
    int rows[2];
    bool valid[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      rows[h] = tile * 16 + 8 * h + g;
      valid[h] = rows[h] < M;
    }
    float acc[NB > 0 ? NB : 1][4];
#pragma unroll
    for (int j = 0; j < (NB > 0 ? NB : 1); ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;

    for (int jc = 0; jc < per; ++jc, ++item) {
      const int kc = warp + jc * W;
      const int k0 = kc * 64 + 16 * c;  // this lane's 16-element segment
      const int s = item % S;
      if (ok) {
        // the outcome is made warp-uniform: the lanes leave together
        ok = __all_sync(0xffffffffu, mbar_wait(&my_bar[s], (item / S) & 1, GWB_ERR_TIMEOUT_ACT));
        if (!ok) failed_at = item;
      }
      float sm[16], rsm[16];
      if (has_smooth) {
        // RN(1 / smooth) of the chunk's 64 columns, two per lane, shared by
        // the warp through shared memory (each column's divide needs it in
        // all 16 rows)
        const uint32_t pair = __ldg(reinterpret_cast<const uint32_t*>(smooth + kc * 64) + lane);
        my_rs[2 * lane] = __frcp_rn(bf_lo(pair));
        my_rs[2 * lane + 1] = __frcp_rn(bf_hi(pair));
        const uint4* sp = reinterpret_cast<const uint4*>(smooth + k0);
        const uint4 s0 = __ldg(sp), s1 = __ldg(sp + 1);
        const uint32_t sw[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          sm[2 * j] = bf_lo(sw[j]);
          sm[2 * j + 1] = bf_hi(sw[j]);
        }
      }
      __syncwarp();
      if (has_smooth) {
        const float4* rp = reinterpret_cast<const float4*>(my_rs + 16 * c);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 r4 = rp[j];
          rsm[4 * j] = r4.x; rsm[4 * j + 1] = r4.y; rsm[4 * j + 2] = r4.z; rsm[4 * j + 3] = r4.w;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) { sm[j] = 1.f; rsm[j] = 1.f; }
      }
      // rows g and g + 8 of the box, 32 bytes each: 16-byte chunks 2c and
      // 2c + 1 of a 128-byte row, at (chunk ^ row % 8) after the swizzle
      uint32_t w[2][8];
      const uint8_t* box = my_xs + s * kBoxBytes;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint8_t* rowp = box + (8 * h + g) * 128;
        const uint4 p0 = *reinterpret_cast<const uint4*>(rowp + (((2 * c) ^ g) << 4));
        const uint4 p1 = *reinterpret_cast<const uint4*>(rowp + (((2 * c + 1) ^ g) << 4));
        w[h][0] = p0.x; w[h][1] = p0.y; w[h][2] = p0.z; w[h][3] = p0.w;
        w[h][4] = p1.x; w[h][5] = p1.y; w[h][6] = p1.z; w[h][7] = p1.w;
      }
      // this chunk's down-projection fragments (L2): the first kEarly rank
      // blocks are requested before the quantisation so their latency hides
      // under it (more would spill), the rest after it
      uint32_t dfr[NB > 0 ? NB : 1][8];
      auto load_dfr = [&](int j) {
        const uint4* dp = reinterpret_cast<const uint4*>(down_t + (size_t)(8 * j + g) * K + k0);
        const uint4 d0 = __ldg(dp), d1 = __ldg(dp + 1);
        dfr[j][0] = d0.x; dfr[j][1] = d0.y; dfr[j][2] = d0.z; dfr[j][3] = d0.w;
        dfr[j][4] = d1.x; dfr[j][5] = d1.y; dfr[j][6] = d1.z; dfr[j][7] = d1.w;
      };
      constexpr int kEarly = NB < 2 ? NB : (NB <= 4 || NB > 8 ? 2 : 0);
#pragma unroll
      for (int j = 0; j < kEarly; ++j) load_dfr(j);
      // every lane has read the box (and the reciprocals): refill the slot
      __syncwarp();
      if (ok) {
        if (lane == 0) fence_proxy_async_smem();
        issue(item + S);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t lo, hi, e23[2];
        __half sc;
        quant_seg16<MMA_FORM>(w[h], sm, rsm, has_smooth, lo, hi, sc, e23);
        if (valid[h]) {
          const int row = rows[h];
          if constexpr (MMA_FORM) {
            *reinterpret_cast<uint4*>(codes + (size_t)row * K + k0) =
                make_uint4(lo, hi, e23[0], e23[1]);
            if (c == 0)
              *reinterpret_cast<uint4*>(ascale + ((size_t)kc * M + row) * 8) =
                  onehot_k8(__half_as_ushort(sc), kc);
          } else {
            *reinterpret_cast<uint2*>(codes + (size_t)row * (K / 2) + k0 / 2) = make_uint2(lo, hi);
            if (c == 0) ascale[(size_t)row * G + kc] = sc;
          }
        }
      }
      if constexpr (NB > 0) {
        // k is permuted consistently in A and B: logical fragment positions
        // (2c,2c+1 | 2c+8,2c+9) of k16-step s map to physical 16c+4s+(0,1 | 2,3).
        // Ranks up to 32 and above 64: the NB accumulators are independent,
        // so step s of every j is issued before step s + 1. Ranks 48 and 64
        // (register-bound) load and consume one rank block at a time.
        if constexpr (kEarly > 0) {
#pragma unroll
          for (int j = kEarly; j < NB; ++j) load_dfr(j);
#pragma unroll
          for (int s4 = 0; s4 < 4; ++s4) {
            const uint32_t a[4] = {w[0][2 * s4], w[1][2 * s4], w[0][2 * s4 + 1],
                                   w[1][2 * s4 + 1]};
#pragma unroll
            for (int j = 0; j < NB; ++j)
              mma_bf16_16816(acc[j], a, dfr[j][2 * s4], dfr[j][2 * s4 + 1]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < NB; ++j) {
            load_dfr(j);
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4) {
              const uint32_t a[4] = {w[0][2 * s4], w[1][2 * s4], w[0][2 * s4 + 1],
                                     w[1][2 * s4 + 1]};
              mma_bf16_16816(acc[j], a, dfr[j][2 * s4], dfr[j][2 * s4 + 1]);
            }
          }
        }
      }
    }

    if constexpr (NB > 0) {
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        float* r0 = red + ((size_t)warp * 16 + g) * RP + 8 * j + 2 * c;
        float* r1 = r0 + 8 * RP;
        r0[0] = acc[j][0];
        r0[1] = acc[j][1];
        r1[0] = acc[j][2];
        r1[1] = acc[j][3];
      }
      __syncthreads();
      for (int i = threadIdx.x; i < 16 * RP; i += blockDim.x) {
        float sum = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < W; ++w2) sum += red[(size_t)w2 * 16 * RP + i];
        const int row = tile * 16 + i / RP;
        if (row < M) la[(size_t)row * RP + i % RP] = __float2bfloat16_rn(sum);
      }
      __syncthreads();
    }
  }
  // after a failed wait: let the boxes still in flight (the one that timed
  // out and any issued after it) land before exiting
  if (!ok && lane == 0)
    for (int i = failed_at; i < issued; ++i) drain_wait(&my_bar[i % S], (i / S) & 1);
}

template <bool MMA_FORM>
static int launch_act_int4_t(const void* x, const void* smooth, const void* down_t, void* codes,
                             void* ascale, void* la, int M, int K, int rank_pad,
                             cudaStream_t st) {
  CUtensorMap tmX;
  int rc = make_tmap(&tmX, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)K, (uint64_t)M, 64,
                     16, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc != GWB_SUCCESS) return rc;
  const int ntiles = (M + 15) / 16;
  const dim3 grid(ntiles < sm_count() ? ntiles : sm_count());
  auto S = static_cast<const __nv_bfloat16*>(smooth);
  auto D = static_cast<const __nv_bfloat16*>(down_t);
  auto C = static_cast<uint8_t*>(codes);
  auto A = static_cast<__half*>(ascale);
  auto L = static_cast<__nv_bfloat16*>(la);
#define GWB_ACT_CASE(RPAD, NBV)                                                              \
  case RPAD: {                                                                               \
    auto k = act_int4_kernel<NBV, MMA_FORM>;                                                 \
    const dim3 block(act_warps<NBV>() * 32);                                                 \
    const size_t smem = actq::smem_bytes<NBV>();                                             \
    static bool attr = false;                                                                \
    if (!attr) {                                                                             \
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);       \
      attr = true;                                                                           \
    }                                                                                        \
    k<<<grid, block, smem, st>>>(tmX, S, D, C, A, L, M, K);                                  \
    break;                                                                                   \
  }
  switch (rank_pad) {
    GWB_ACT_CASE(0, 0)
    GWB_ACT_CASE(16, 2)
    GWB_ACT_CASE(32, 4)
    GWB_ACT_CASE(48, 6)
    GWB_ACT_CASE(64, 8)
    GWB_ACT_CASE(80, 10)
    GWB_ACT_CASE(96, 12)
    GWB_ACT_CASE(112, 14)
    GWB_ACT_CASE(128, 16)
    default: return GWB_E_SHAPE;
  }
#undef GWB_ACT_CASE
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

int launch_act_int4(const void* x, const void* smooth, const void* down_t, void* codes,
                    void* ascale, void* la, int M, int K, int rank_pad, bool mma_form,
                    cudaStream_t st) {
  if (M <= 0 || K <= 0 || K % 64) return GWB_E_SHAPE;
  if (mma_form)
    return launch_act_int4_t<true>(x, smooth, down_t, codes, ascale, la, M, K, rank_pad, st);
  return launch_act_int4_t<false>(x, smooth, down_t, codes, ascale, la, M, K, rank_pad, st);
}

// Scale interchange form f16 [R, K/64] -> GEMM scale-operand rows
// f16 [K/64, R, 8] (group g's scale at k = g mod 8, zeros elsewhere).
__global__ void scale_k8_kernel(const __half* __restrict__ scale, uint4* __restrict__ scale_k8,
                                int R, int G) {
  const int64_t n = (int64_t)R * G;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / G, g = i % G;
    scale_k8[(size_t)g * R + r] = onehot_k8(__half_as_ushort(scale[i]), (int)g);
  }
}

int launch_scale_k8(const void* scale, void* scale_k8, int R, int K, cudaStream_t st) {
  if (R <= 0 || K <= 0 || K % 64) return GWB_E_SHAPE;
  const int64_t work = (int64_t)R * (K / 64);
  int64_t blocks = (work + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  scale_k8_kernel<<<(int)blocks, 256, 0, st>>>(static_cast<const __half*>(scale),
                                               static_cast<uint4*>(scale_k8), R, K / 64);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

// One warp per row: pass 1 amax, pass 2 (L1/L2-resident re-read) quantise.
__global__ void __launch_bounds__(256)
act_int8_kernel(const __nv_bfloat16* __restrict__ x, int8_t* __restrict__ q,
                float* __restrict__ scale, int M, int K) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= M) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)warp * K);
  const int nvec = K / 8;
  float amax = 0.f;
  for (int i = lane; i < nvec; i += 32) {
    uint4 p = __ldg(xr + i);
    uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) amax = fmaxf(amax, fmaxf(fabsf(bf_lo(w[j])), fabsf(bf_hi(w[j]))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = fmaxf(__fdiv_rn(amax, 127.0f), 1e-12f);
  if (lane == 0) scale[warp] = s;
  uint2* qr = reinterpret_cast<uint2*>(q + (size_t)warp * K);
  for (int i = lane; i < nvec; i += 32) {
    uint4 p = __ldg(xr + i);
    uint32_t w[4] = {p.x, p.y, p.z, p.w};
    uint32_t packed[2] = {0, 0};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a = fminf(fmaxf(rintf(__fdiv_rn(bf_lo(w[j]), s)), -127.f), 127.f);
      float b = fminf(fmaxf(rintf(__fdiv_rn(bf_hi(w[j]), s)), -127.f), 127.f);
      uint32_t qa = static_cast<uint32_t>(static_cast<int>(a)) & 0xFFu;
      uint32_t qb = static_cast<uint32_t>(static_cast<int>(b)) & 0xFFu;
      packed[j >> 1] |= (qa | (qb << 8)) << (16 * (j & 1));
    }
    qr[i] = make_uint2(packed[0], packed[1]);
  }
}

int launch_act_int8(const void* x, void* q, void* scale, int M, int K, cudaStream_t st) {
  const int warps_per_block = 8;
  dim3 grid((M + warps_per_block - 1) / warps_per_block), block(warps_per_block * 32);
  act_int8_kernel<<<grid, block, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                          static_cast<int8_t*>(q), static_cast<float*>(scale),
                                          M, K);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

// FP8 (e4m3) rowwise, one warp per row as act_int8_kernel: the dynamic
// rowwise branch of the reference's _quant_src
// (src/gen_worker/models/w8a8.py:261-273): sa = max(amax / 448, 1e-12) in
// f32; the reciprocal 1/sa (f32) rounded to bf16; q = e4m3(clamp(bf16(x *
// inv), +-448)), round-to-nearest-even with subnormals. x * inv is exact in
// f32 (two 8-bit significands), so its bf16 rounding matches a bf16 multiply.
__global__ void __launch_bounds__(256)
act_fp8_kernel(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ q,
               float* __restrict__ scale, int M, int K) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= M) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)warp * K);
  const int nvec = K / 8;
  float amax = 0.f;
  for (int i = lane; i < nvec; i += 32) {
    uint4 p = __ldg(xr + i);
    uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) amax = fmaxf(amax, fmaxf(fabsf(bf_lo(w[j])), fabsf(bf_hi(w[j]))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = fmaxf(__fdiv_rn(amax, 448.0f), 1e-12f);
  if (lane == 0) scale[warp] = s;
  const float inv = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(1.0f, s)));
  uint2* qr = reinterpret_cast<uint2*>(q + (size_t)warp * K);
  for (int i = lane; i < nvec; i += 32) {
    uint4 p = __ldg(xr + i);
    uint32_t w[4] = {p.x, p.y, p.z, p.w};
    uint32_t packed[2] = {0, 0};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 v;
      v.x = fminf(fmaxf(__bfloat162float(__float2bfloat16_rn(bf_lo(w[j]) * inv)), -448.f), 448.f);
      v.y = fminf(fmaxf(__bfloat162float(__float2bfloat16_rn(bf_hi(w[j]) * inv)), -448.f), 448.f);
      const uint32_t pair = __nv_cvt_float2_to_fp8x2(v, __NV_SATFINITE, __NV_E4M3);
      packed[j >> 1] |= (pair & 0xFFFFu) << (16 * (j & 1));
    }
    qr[i] = make_uint2(packed[0], packed[1]);
  }
}

// ------------------------------------------------------------------ NVFP4
// The reference's NVFP4 activation quantiser (quantize_activation_torch,
// src/gen_worker/models/nvfp4_quant.py:92-103), after the smoothing divide
// and the per-tensor second-level scale of SvdqLinear.forward
// (svdq_native.py:144-146).
//   work f32 [4 + K] (16-byte aligned): [0] amax (fp32 bits), [1] s2,
//   [4, 4 + K) = RN(1 / smooth) (16-byte aligned for float4 reads).
//   nvfp4_rsmooth_kernel: the smoothing reciprocals, once per call.
//   nvfp4_amax_kernel: amax |bf16(x / smooth)| over the whole tensor (fp32
//     bits, atomicMax; the values are non-negative) into work[0].
//   act_nvfp4_kernel: s2 = max(amax / 2688, 1e-12) (written to work[1]);
//     per 16-block: sa = e4m3(clamp(bmax / (6 s2), 2^-9, 448)) (nearest-
//     even), q = xs / (sa * s2) (fp32, correctly rounded), e2m1 code with the
//     reference's tie rule (cast_e2m1, nvfp4_quant.py:41-51); codes packed
//     with element 2j in the low nibble, scales written at their cuBLAS
//     blocked-layout address (to_blocked_scales, nvfp4_quant.py:72-84).

// bf16(x / smooth) for 8 packed bf16 at column c8 (reciprocals from rsm)
__device__ __forceinline__ void smooth8(const uint4& xv, const uint4& sv, const float* rsm,
                                        float (&o)[8]) {
  const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
  const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
  const float4 r0 = *reinterpret_cast<const float4*>(rsm);
  const float4 r1 = *reinterpret_cast<const float4*>(rsm + 4);
  const float rr[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    o[2 * j] = __bfloat162float(__float2bfloat16_rn(div_rn(bf_lo(xw[j]), bf_lo(sw[j]), rr[2 * j])));
    o[2 * j + 1] =
        __bfloat162float(__float2bfloat16_rn(div_rn(bf_hi(xw[j]), bf_hi(sw[j]), rr[2 * j + 1])));
  }
}

__global__ void nvfp4_rsmooth_kernel(const __nv_bfloat16* __restrict__ smooth,
                                     float* __restrict__ rsm, int K) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < K) rsm[i] = __frcp_rn(__bfloat162float(smooth[i]));
}

__device__ __forceinline__ void raw8(const uint4& xv, float (&o)[8]) {
  const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) { o[2 * j] = bf_lo(xw[j]); o[2 * j + 1] = bf_hi(xw[j]); }
}

__global__ void __launch_bounds__(256)
nvfp4_amax_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ smooth,
                  const float* __restrict__ rsm, unsigned int* __restrict__ amax_bits, int M,
                  int K) {
  const int64_t nvec = (int64_t)M * K / 8;
  const int kv = K / 8;
  float m = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nvec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x) + i);
    float v[8];
    const int cv = (int)(i % kv);
    if (smooth) smooth8(xv, __ldg(reinterpret_cast<const uint4*>(smooth) + cv), rsm + 8 * cv, v);
    else raw8(xv, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(v[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) b = fmaxf(b, red[w]);
    atomicMax(amax_bits, __float_as_uint(b));
  }
}

// e2m1 magnitude code of |q| with the reference's rounding: the number of the
// bounds 0.25 0.75 1.25 1.75 2.5 3.5 5.0 strictly below |q|, plus one when
// |q| is exactly 0.75, 1.75 or 2.5.
// (sign bit set when q < 0.) Two such codes (a in the low nibble) come from
// the hardware conversion: cvt.rn.satfinite.e2m1x2.f32 rounds to nearest-even and
// saturates at 6, which is the rule above except at the ties |q| = 2.5 and
// 3.5 (the reference takes 3.0 for both, nearest-even takes 2.0 and 4.0) and
// at q = -0 (the reference sets no sign bit); those three cases are patched.
__device__ __forceinline__ uint32_t e2m1x2_code(float a, float b) {
  a = __fadd_rn(a, 0.0f);   // -0 -> +0
  b = __fadd_rn(b, 0.0f);
  uint32_t r;
  asm("{ .reg .b8 t;\n\t cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t cvt.u32.u8 %0, t;\n\t}"
      : "=r"(r) : "f"(b), "f"(a));
  const float aa = fabsf(a), ab = fabsf(b);
  if (aa == 2.5f || aa == 3.5f) r = (r & 0xF0u) | 5u | (a < 0.0f ? 8u : 0u);
  if (ab == 2.5f || ab == 3.5f) r = (r & 0x0Fu) | ((5u | (b < 0.0f ? 8u : 0u)) << 4);
  return r;
}

__global__ void __launch_bounds__(256)
act_nvfp4_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ smooth,
                 float* __restrict__ work, uint8_t* __restrict__ codes,
                 uint8_t* __restrict__ sblk, int M, int K,
                 __nv_bfloat16* __restrict__ la3 = nullptr, int rank_pad = 0) {
  const float amax = __uint_as_float(*reinterpret_cast<const volatile unsigned int*>(work));
  const float s2 = fmaxf(__fdiv_rn(amax, 6.0f * 448.0f), 1e-12f);
  if (blockIdx.x == 0 && threadIdx.x == 0) work[1] = s2;
  if (la3 != nullptr) {
    // la3 row = [u_hi | u_lo | u_hi], u = la / s2 (la = bf16(x · proj_down),
    // in columns [0, rank_pad) of the row); one thread owns each (row, j)
    const int64_t nla = (int64_t)M * rank_pad;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nla;
         i += (int64_t)gridDim.x * blockDim.x) {
      __nv_bfloat16* r = la3 + (i / rank_pad) * 3 * rank_pad;
      const int j = (int)(i % rank_pad);
      const float u = __fdiv_rn(__bfloat162float(r[j]), s2);
      const __nv_bfloat16 uh = __float2bfloat16_rn(u);
      const __nv_bfloat16 ul = __float2bfloat16_rn(u - __bfloat162float(uh));
      r[j] = uh;
      r[rank_pad + j] = ul;
      r[2 * rank_pad + j] = uh;
    }
  }
  const float d6 = 6.0f * s2;
  const int kb16 = K / 16;
  const int ncb = (kb16 + 3) / 4;
  const int64_t nblk = (int64_t)M * kb16;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < nblk;
       b += (int64_t)gridDim.x * blockDim.x) {
    const int row = (int)(b / kb16), c = (int)(b % kb16);
    const uint4* xp = reinterpret_cast<const uint4*>(x + (size_t)row * K + c * 16);
    float v[16];
    float lo[8], hi[8];
    if (smooth) {
      const uint4* sp = reinterpret_cast<const uint4*>(smooth + c * 16);
      smooth8(__ldg(xp), __ldg(sp), work + 4 + c * 16, lo);
      smooth8(__ldg(xp + 1), __ldg(sp + 1), work + 4 + c * 16 + 8, hi);
    } else {
      raw8(__ldg(xp), lo);
      raw8(__ldg(xp + 1), hi);
    }
    float bmax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = lo[j];
      v[8 + j] = hi[j];
      bmax = fmaxf(bmax, fmaxf(fabsf(lo[j]), fabsf(hi[j])));
    }
    const float t = fminf(fmaxf(__fdiv_rn(bmax, d6), 0.001953125f), 448.0f);
    const uint32_t sbyte = __nv_cvt_float_to_fp8(t, __NV_SATFINITE, __NV_E4M3) & 0xFFu;
    const __half_raw hr = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)sbyte, __NV_E4M3);
    const float sa = __half2float(__half(hr));
    const float den = sa * s2;
    const float rden = __frcp_rn(den);
    uint32_t w0 = 0, w1 = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      w0 |= e2m1x2_code(div_rn(v[2 * j], den, rden), div_rn(v[2 * j + 1], den, rden)) << (8 * j);
      w1 |= e2m1x2_code(div_rn(v[8 + 2 * j], den, rden), div_rn(v[9 + 2 * j], den, rden))
            << (8 * j);
    }
    *reinterpret_cast<uint2*>(codes + (size_t)row * (K / 2) + c * 8) = make_uint2(w0, w1);
    const size_t off = ((size_t)(row >> 7) * ncb + (c >> 2)) * 512 + (row & 31) * 16 +
                       ((row & 127) >> 5) * 4 + (c & 3);
    sblk[off] = (uint8_t)sbyte;
  }
  // zero scales of the padding rows up to the next multiple of 128 (the
  // reference's to_blocked_scales pads with zeros)
  const int mpad = ((M + 127) / 128) * 128;
  const int64_t npad = (int64_t)(mpad - M) * kb16;
  for (int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; b < npad;
       b += (int64_t)gridDim.x * blockDim.x) {
    const int row = M + (int)(b / kb16), c = (int)(b % kb16);
    sblk[((size_t)(row >> 7) * ncb + (c >> 2)) * 512 + (row & 31) * 16 +
         ((row & 127) >> 5) * 4 + (c & 3)] = 0;
  }
}

// amax |bf16(x / smooth)| (as nvfp4_amax_kernel) fused with the low-rank
// down-projection la = bf16(x · L1) on RAW x (written to the first rank_pad
// columns of the [M, 3 * rank_pad] la3 rows; act_nvfp4_kernel then splits it), so the NVFP4 lane reads x twice
// per call (this pass and the quantiser) instead of three times. Layout and
// MMA fragments as act_int4_kernel: 16 rows per CTA, 8 warps splitting K in
// 64-wide chunks, lane (g, c) on rows g and g + 8 and the 16 columns
// 64 kc + 16 c; k is permuted alike in the x and L1 fragments (logical
// positions (2c, 2c+1 | 2c+8, 2c+9) of k16-step s are physical
// 16c + 4s + (0, 1 | 2, 3)); the per-warp partial sums of la are added in a
// fixed order through shared memory (deterministic).
template <int NB>
__global__ void __launch_bounds__(256, NB > 8 ? 1 : 2)
nvfp4_amax_la_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ smooth,
                     const float* __restrict__ rsm, const __nv_bfloat16* __restrict__ down_t,
                     unsigned int* __restrict__ amax_bits, __nv_bfloat16* __restrict__ la, int M,
                     int K) {
  constexpr int RP = NB * 8, ROWS = 16, WARPS = 8;
  // per-warp partial sums of la: [WARPS][ROWS][RP] floats (64 KB at rank 128,
  // beyond the static limit, hence dynamic)
  extern __shared__ float red_dyn[];
  float (*red)[ROWS][RP] = reinterpret_cast<float (*)[ROWS][RP]>(red_dyn);
  __shared__ float wmax[WARPS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int nchunks = K / 64;
  int rows[2];
  bool valid[2];
  const uint4* xr[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    rows[h] = blockIdx.x * ROWS + 8 * h + g;
    valid[h] = rows[h] < M;
    xr[h] = reinterpret_cast<const uint4*>(x + (size_t)(valid[h] ? rows[h] : 0) * K);
  }
  float acc[NB][4];
#pragma unroll
  for (int j = 0; j < NB; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
  float m = 0.f;
  for (int kc = warp; kc < nchunks; kc += WARPS) {
    const int k0 = kc * 64 + 16 * c;
    uint32_t w[2][8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 p0 = valid[h] ? __ldg(xr[h] + k0 / 8) : make_uint4(0, 0, 0, 0);
      const uint4 p1 = valid[h] ? __ldg(xr[h] + k0 / 8 + 1) : make_uint4(0, 0, 0, 0);
      w[h][0] = p0.x; w[h][1] = p0.y; w[h][2] = p0.z; w[h][3] = p0.w;
      w[h][4] = p1.x; w[h][5] = p1.y; w[h][6] = p1.z; w[h][7] = p1.w;
      float v[8];
      if (smooth) {
        smooth8(p0, __ldg(reinterpret_cast<const uint4*>(smooth + k0)), rsm + k0, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(v[e]));
        smooth8(p1, __ldg(reinterpret_cast<const uint4*>(smooth + k0) + 1), rsm + k0 + 8, v);
      } else {
        raw8(p0, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(v[e]));
        raw8(p1, v);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(v[e]));
    }
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      const uint4* dp = reinterpret_cast<const uint4*>(down_t + (size_t)(8 * j + g) * K + k0);
      const uint4 d0 = __ldg(dp), d1 = __ldg(dp + 1);
      const uint32_t dw[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const uint32_t a[4] = {w[0][2 * s], w[1][2 * s], w[0][2 * s + 1], w[1][2 * s + 1]};
        mma_bf16_16816(acc[j], a, dw[2 * s], dw[2 * s + 1]);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) wmax[warp] = m;
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    red[warp][g][8 * j + 2 * c] = acc[j][0];
    red[warp][g][8 * j + 2 * c + 1] = acc[j][1];
    red[warp][g + 8][8 * j + 2 * c] = acc[j][2];
    red[warp][g + 8][8 * j + 2 * c + 1] = acc[j][3];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = wmax[0];
    for (int w2 = 1; w2 < WARPS; ++w2) b = fmaxf(b, wmax[w2]);
    atomicMax(amax_bits, __float_as_uint(b));
  }
  for (int i = threadIdx.x; i < ROWS * RP; i += blockDim.x) {
    const int r = i / RP, col = i % RP;
    float sum = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < WARPS; ++w2) sum += red[w2][r][col];
    const int row = blockIdx.x * ROWS + r;
    if (row < M) la[(size_t)row * (3 * RP) + col] = __float2bfloat16_rn(sum);
  }
}

int launch_act_nvfp4(const void* x, const void* smooth, float* work, void* codes, void* sblk,
                     int M, int K, cudaStream_t st) {
  if (cudaMemsetAsync(work, 0, sizeof(float), st) != cudaSuccess) return GWB_E_LAUNCH;
  if (smooth)
    nvfp4_rsmooth_kernel<<<(K + 255) / 256, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(smooth), work + 4, K);
  const int64_t nvec = (int64_t)M * K / 8;
  int64_t blocks = (nvec + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  nvfp4_amax_kernel<<<(int)blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                                  static_cast<const __nv_bfloat16*>(smooth),
                                                  work + 4, reinterpret_cast<unsigned int*>(work),
                                                  M, K);
  const int64_t nblk = (int64_t)M * (K / 16);
  blocks = (nblk + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  act_nvfp4_kernel<<<(int)blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                                 static_cast<const __nv_bfloat16*>(smooth), work,
                                                 static_cast<uint8_t*>(codes),
                                                 static_cast<uint8_t*>(sblk), M, K);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

int launch_act_nvfp4_lowrank(const void* x, const void* smooth, const void* down_t, float* work,
                             void* codes, void* sblk, void* la, int M, int K, int rank_pad,
                             cudaStream_t st) {
  if (cudaMemsetAsync(work, 0, sizeof(float), st) != cudaSuccess) return GWB_E_LAUNCH;
  if (smooth)
    nvfp4_rsmooth_kernel<<<(K + 255) / 256, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(smooth), work + 4, K);
  const dim3 grid((M + 15) / 16);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto Sm = static_cast<const __nv_bfloat16*>(smooth);
  auto D = static_cast<const __nv_bfloat16*>(down_t);
  auto A = reinterpret_cast<unsigned int*>(work);
  auto L = static_cast<__nv_bfloat16*>(la);
  const size_t red_bytes = (size_t)8 * 16 * rank_pad * sizeof(float);
#define GWB_AMAX_LA_CASE(RPAD, NBV)                                                          \
  case RPAD: {                                                                               \
    auto k = nvfp4_amax_la_kernel<NBV>;                                                      \
    if (red_bytes > 48 * 1024)                                                               \
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)red_bytes);  \
    k<<<grid, 256, red_bytes, st>>>(X, Sm, work + 4, D, A, L, M, K);                          \
    break;                                                                                   \
  }
  switch (rank_pad) {
    GWB_AMAX_LA_CASE(16, 2)
    GWB_AMAX_LA_CASE(32, 4)
    GWB_AMAX_LA_CASE(48, 6)
    GWB_AMAX_LA_CASE(64, 8)
    GWB_AMAX_LA_CASE(80, 10)
    GWB_AMAX_LA_CASE(96, 12)
    GWB_AMAX_LA_CASE(112, 14)
    GWB_AMAX_LA_CASE(128, 16)
    default: return GWB_E_SHAPE;
  }
#undef GWB_AMAX_LA_CASE
  const int64_t nblk = (int64_t)M * (K / 16);
  int64_t blocks = (nblk + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  act_nvfp4_kernel<<<(int)blocks, 256, 0, st>>>(X, Sm, work, static_cast<uint8_t*>(codes),
                                                 static_cast<uint8_t*>(sblk), M, K, L, rank_pad);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

int launch_act_fp8(const void* x, void* q, void* scale, int M, int K, cudaStream_t st) {
  const int warps_per_block = 8;
  dim3 grid((M + warps_per_block - 1) / warps_per_block), block(warps_per_block * 32);
  act_fp8_kernel<<<grid, block, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                         static_cast<uint8_t*>(q), static_cast<float*>(scale),
                                         M, K);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

}  // namespace gwb
