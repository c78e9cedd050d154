// AWQ W4A16 modulation GEMV (the reference's `cozy_gen_worker::awq_w4a16_mm`,
// src/gen_worker/models/svdq_awq_packed.py:51-103): y[m, n] = sum_k x[m, k] *
// bf16(q[n, k] * wscales[n, g] + wzeros[n, g]) + bias[n], g = k / 64, with
// unsigned 4-bit codes packed two per byte (even k in the low nibble),
// wscales / wzeros bf16 [N, K/64] (zeros pre-scaled and pre-negated), f32
// accumulation, bf16 output.
//
// The layers are the timestep-embedding modulations: M is the batch (1-2),
// N up to 18432, K = 3072: the codes are streamed once from HBM (16-byte
// loads) and the kernel must keep the issue slots below the HBM time. Per
// pair of codes it spends a byte permute and one LOP3 (both nibbles of a byte
// placed under the bf16 exponent of 128), a bf16x2 subtract that recovers the
// codes exactly and one bf16x2 FMA forming q * s + z, and leaves the dot
// product to the tensor cores: one mma.sync m16n8k16 per 16 codes of 16 weight
// rows, the dequantised weight as the A operand and x (the batch, up to 8
// rows per CTA) as B. The FP32
// pipe is not used (its FFMA2 rate bounded a scalar-dequant version at
// ~1.6 TB/s). mma.sync suffices: the GEMV is memory bound and needs no TMEM
// accumulator. Each CTA covers 16 weight rows with K split over its 8 warps,
// so a warp holds the loads of three 128-code superchunks in flight at once.
//
// Rounding: q * s is exact (4 x 8 significant bits) and the bf16 FMA rounds
// q * s + z once. The reference rounds it to f32 and then to bf16; the two
// agree whenever q * s + z fits 24 significant bits, which holds for AWQ's
// grids (|z| is the group minimum, within 15 s of every q * s), and differ by
// one bf16 unit in the last place otherwise.
#include <cuda_bf16.h>
#include <cstdint>

namespace gwb {
namespace awq {

#ifndef GWB_AWQ_WARPS
#define GWB_AWQ_WARPS 8
#endif
#ifndef GWB_AWQ_UNROLL
#define GWB_AWQ_UNROLL 3
#endif
constexpr int WARPS = GWB_AWQ_WARPS;   // warps per CTA, splitting K
constexpr int TILES = 2;               // 8-row weight tiles per CTA tile (16 output rows)
constexpr int UNROLL = GWB_AWQ_UNROLL; // superchunks per warp whose loads are issued together
constexpr int SC = 128;       // codes per superchunk (one 16-byte load per lane and row)
constexpr int MT = 8;         // batch rows per CTA (the MMA's B columns)

// bf16x2 (128 + code of the low nibble of byte i of w, 128 + code of its
// high nibble): byte i of w lands in byte 0, byte i of w >> 4 in byte 2, the
// nibbles are kept at bits 0-3 / 16-19 and the exponent of 128 is set.
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, uint32_t w4, int i) {
  const uint32_t p = __byte_perm(w, w4, (uint32_t)(i | ((4 + i) << 8)));
  return (p & 0x000F000Fu) | 0x43004300u;
}

// q * s + z for a pair of codes, in bf16 with one rounding (fma.rn.bf16x2).
__device__ __forceinline__ uint32_t dequant_pair(uint32_t biased, __nv_bfloat162 s2,
                                                 __nv_bfloat162 z2) {
  const __nv_bfloat162 c128 = __floats2bfloat162_rn(128.0f, 128.0f);
  const __nv_bfloat162 q = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&biased), c128);
  const __nv_bfloat162 w = __hfma2(q, s2, z2);
  return *reinterpret_cast<const uint32_t*>(&w);
}

// One CTA: TILES x 8 = 16 weight rows against a tile of up to MT = 8 batch
// rows, K split over the WARPS warps (warp w takes superchunks w, w + WARPS,
// ...), partial sums reduced through shared memory. Lane (g, t) = (lane / 4,
// lane % 4) streams bytes [16 t, 16 t + 16) of each 128-code superchunk of
// weight rows n0 + g and n0 + 8 + g: 16 code pairs per row. Each mma.sync
// m16n8k16 takes the 16 weight rows as A (rows g and g + 8 of the fragment)
// and the batch as B (column g = batch row m0 + g), so one MMA covers 16
// codes of all 16 weight rows. MMA slice s (16 codes) takes the lane's
// pairs 2s (k-slots 2t, 2t + 1) and 2s + 1 (k-slots 2t + 8, 2t + 9) of both
// rows; x is read at the same code positions (32 consecutive bf16 per lane
// and batch row), so every slice is a 16-term dot product over codes of the
// superchunk. Each warp issues the loads of UNROLL superchunks before their
// arithmetic.
__global__ void __launch_bounds__(WARPS * 32)
awq_w4a16_kernel(const __nv_bfloat16* __restrict__ x, const uint8_t* __restrict__ w,
                 const __nv_bfloat16* __restrict__ ws, const __nv_bfloat16* __restrict__ wz,
                 const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ out,
                 int M, int N, int K) {
  __shared__ float red[WARPS][4][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int n0 = blockIdx.x * TILES * 8;
  const int m0 = blockIdx.y * MT;
  const int G = K / 64, nsc = K / SC;
  const bool xa = m0 + g < M;
  const uint4* xra = reinterpret_cast<const uint4*>(x + (size_t)(xa ? m0 + g : 0) * K) + 4 * t;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};

  for (int sc0 = warp; sc0 < nsc; sc0 += WARPS * UNROLL) {
    uint4 wv[UNROLL][TILES];
    __nv_bfloat162 s2[UNROLL][TILES], z2[UNROLL][TILES];
    uint4 xv[UNROLL][4];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int sc = sc0 + u * WARPS;
      const bool live = sc < nsc;
#pragma unroll
      for (int i = 0; i < TILES; ++i) {
        const int n = min(n0 + 8 * i + g, N - 1);
        const int grp = sc * 2 + (t >> 1);
        if (live) {
          wv[u][i] = __ldcs(reinterpret_cast<const uint4*>(w + (size_t)n * (K / 2) + sc * (SC / 2)) + t);
          s2[u][i] = __bfloat162bfloat162(ws[(size_t)n * G + grp]);
          z2[u][i] = __bfloat162bfloat162(wz[(size_t)n * G + grp]);
        } else {
          wv[u][i] = make_uint4(0, 0, 0, 0);
          s2[u][i] = z2[u][i] = __bfloat162bfloat162(__float2bfloat16(0.f));
        }
      }
#pragma unroll
      for (int h = 0; h < 4; ++h)
        xv[u][h] = (live && xa) ? __ldg(xra + sc * (SC / 8) + h) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const uint32_t* xa32 = reinterpret_cast<const uint32_t*>(&xv[u][0]);
      const uint32_t w0[4] = {wv[u][0].x, wv[u][0].y, wv[u][0].z, wv[u][0].w};
      const uint32_t w1[4] = {wv[u][1].x, wv[u][1].y, wv[u][1].z, wv[u][1].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t w0s = w0[q] >> 4, w1s = w1[q] >> 4;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          // slice s = 2q + h: pairs 2s and 2s + 1 = bytes 2h and 2h + 1 of word q
          const int sl = 2 * q + h;
          const uint32_t a[4] = {dequant_pair(nib_pair(w0[q], w0s, 2 * h), s2[u][0], z2[u][0]),
                                 dequant_pair(nib_pair(w1[q], w1s, 2 * h), s2[u][1], z2[u][1]),
                                 dequant_pair(nib_pair(w0[q], w0s, 2 * h + 1), s2[u][0], z2[u][0]),
                                 dequant_pair(nib_pair(w1[q], w1s, 2 * h + 1), s2[u][1], z2[u][1])};
          mma_bf16_16816(acc, a, xa32[2 * sl], xa32[2 * sl + 1]);
        }
      }
    }
  }
  // split-K reduction: acc = D[g][2t, 2t + 1] and D[g + 8][2t, 2t + 1]
  // (weight rows n0 + g (+ 8), batch rows m0 + 2t (+ 1))
#pragma unroll
  for (int e = 0; e < 4; ++e) red[warp][e][lane] = acc[e];
  __syncthreads();
  if (warp != 0) return;
  float v[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    v[e] = 0.f;
#pragma unroll
    for (int ww = 0; ww < WARPS; ++ww) v[e] += red[ww][e][lane];
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int n = n0 + g + 8 * (e >> 1), m = m0 + 2 * t + (e & 1);
    if (m < M) {
      const float b = bias != nullptr ? __bfloat162float(bias[n]) : 0.f;
      out[(size_t)m * N + n] = __float2bfloat16_rn(v[e] + b);
    }
  }
}

}  // namespace awq

// Grid: one CTA per 16 weight rows x 8 batch rows. Requires N % 16 == 0,
// K % 128 == 0, 16-byte aligned x / w.
inline cudaError_t launch_awq_w4a16(const __nv_bfloat16* x, const uint8_t* w,
                                    const __nv_bfloat16* ws, const __nv_bfloat16* wz,
                                    const __nv_bfloat16* bias, __nv_bfloat16* out, int M,
                                    int N, int K, cudaStream_t st) {
  using namespace awq;
  dim3 grid(N / (TILES * 8), (M + MT - 1) / MT);
  awq_w4a16_kernel<<<grid, WARPS * 32, 0, st>>>(x, w, ws, wz, bias, out, M, N, K);
  return cudaGetLastError();
}

}  // namespace gwb
