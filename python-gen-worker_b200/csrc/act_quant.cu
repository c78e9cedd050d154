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
#include <cstdint>
#include "gwb.h"
#include "ptx.cuh"

namespace gwb {

constexpr int kActRows = 16;    // rows per CTA (one m16 MMA tile)
constexpr int kActWarps = 8;    // warps per CTA, splitting K round-robin

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// sign-magnitude nibble of clamp(rint(v/s), -7, 7): bit 3 = sign, bits 0-2 = |q|
__device__ __forceinline__ uint32_t q4(float v, float s) {
  float q = rintf(__fdiv_rn(v, s));
  q = fminf(fmaxf(q, -7.0f), 7.0f);
  const int qi = static_cast<int>(q);
  return qi < 0 ? (8u | static_cast<uint32_t>(-qi)) : static_cast<uint32_t>(qi);
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Quantise 16 consecutive raw elements (8 bf16x2 words) of one row-group
// segment. The 4 lanes of a quad hold the 64 elements of one group.
__device__ __forceinline__ void quant_seg16(const uint32_t (&xw)[8], const uint32_t (&sw)[8],
                                            bool has_smooth, uint32_t& lo, uint32_t& hi,
                                            __half& scale_out) {
  float v[16];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float a = bf_lo(xw[j]), b = bf_hi(xw[j]);
    if (has_smooth) {
      a = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(a, bf_lo(sw[j]))));
      b = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(b, bf_hi(sw[j]))));
    }
    v[2 * j] = a;
    v[2 * j + 1] = b;
  }
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
  float s32 = __fdiv_rn(amax, 7.0f);
  s32 = fminf(fmaxf(s32, 5.9604644775390625e-08f), 65504.0f);
  __half sh = __float2half_rn(s32);
  float s = __half2float(sh);
  lo = 0;
  hi = 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) lo |= q4(v[j], s) << (4 * j);
#pragma unroll
  for (int j = 0; j < 8; ++j) hi |= q4(v[8 + j], s) << (4 * j);
  scale_out = sh;
}

// NB = padded rank / 8 (0 = no low-rank branch). MMA_FORM = false writes the
// interchange form: packed codes u8 [M, K/2] and ascale f16 [M, K/64].
// MMA_FORM = true writes the GEMM operand form: codes u8 [M, K] as e4m3
// bytes of q * 2^-9 in the within-8 operand order (unpack8_e4m3), and the
// scales as scale-operand rows f16 [K/64, M, 8] (scale at k = 0, zeros at
// k = 1..7: one 16-byte TMA row per matrix row).
template <int NB, bool MMA_FORM>
__global__ void __launch_bounds__(kActWarps * 32)
act_int4_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ smooth,
                const __nv_bfloat16* __restrict__ down_t, uint8_t* __restrict__ codes,
                __half* __restrict__ ascale, __nv_bfloat16* __restrict__ la, int M, int K) {
  constexpr int RP = NB * 8;
  __shared__ float red[NB > 0 ? kActWarps : 1][kActRows][RP > 0 ? RP : 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int row0 = blockIdx.x * kActRows + g, row1 = row0 + 8;
  const bool v0 = row0 < M, v1 = row1 < M;
  const int nchunks = K / 64;
  const int G = K / 64;

  float acc[NB > 0 ? NB : 1][4];
#pragma unroll
  for (int j = 0; j < (NB > 0 ? NB : 1); ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[j][e] = 0.f;

  const uint4* xr0 = reinterpret_cast<const uint4*>(x + (size_t)(v0 ? row0 : 0) * K);
  const uint4* xr1 = reinterpret_cast<const uint4*>(x + (size_t)(v1 ? row1 : 0) * K);

  for (int kc = warp; kc < nchunks; kc += kActWarps) {
    const int k0 = kc * 64 + 16 * c;  // this lane's 16-element segment
    uint32_t w0[8], w1[8];
    {
      uint4 p0 = v0 ? __ldg(xr0 + k0 / 8) : make_uint4(0, 0, 0, 0);
      uint4 p1 = v0 ? __ldg(xr0 + k0 / 8 + 1) : make_uint4(0, 0, 0, 0);
      uint4 q0 = v1 ? __ldg(xr1 + k0 / 8) : make_uint4(0, 0, 0, 0);
      uint4 q1 = v1 ? __ldg(xr1 + k0 / 8 + 1) : make_uint4(0, 0, 0, 0);
      w0[0] = p0.x; w0[1] = p0.y; w0[2] = p0.z; w0[3] = p0.w;
      w0[4] = p1.x; w0[5] = p1.y; w0[6] = p1.z; w0[7] = p1.w;
      w1[0] = q0.x; w1[1] = q0.y; w1[2] = q0.z; w1[3] = q0.w;
      w1[4] = q1.x; w1[5] = q1.y; w1[6] = q1.z; w1[7] = q1.w;
    }
    uint32_t sw[8];
    const bool has_smooth = smooth != nullptr;
    if (has_smooth) {
      const uint4* sp = reinterpret_cast<const uint4*>(smooth + k0);
      uint4 s0 = __ldg(sp), s1 = __ldg(sp + 1);
      sw[0] = s0.x; sw[1] = s0.y; sw[2] = s0.z; sw[3] = s0.w;
      sw[4] = s1.x; sw[5] = s1.y; sw[6] = s1.z; sw[7] = s1.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) sw[j] = 0;
    }
    uint32_t lo0, hi0, lo1, hi1;
    __half s0, s1;
    quant_seg16(w0, sw, has_smooth, lo0, hi0, s0);
    quant_seg16(w1, sw, has_smooth, lo1, hi1, s1);
    if (v0) {
      if constexpr (MMA_FORM) {
        uint4 o;
        unpack8_e4m3(lo0, o.x, o.y);
        unpack8_e4m3(hi0, o.z, o.w);
        *reinterpret_cast<uint4*>(codes + (size_t)row0 * K + k0) = o;
      } else {
        *reinterpret_cast<uint2*>(codes + (size_t)row0 * (K / 2) + k0 / 2) = make_uint2(lo0, hi0);
      }
      if (c == 0) {
        if constexpr (MMA_FORM)
          *reinterpret_cast<uint4*>(ascale + ((size_t)kc * M + row0) * 8) =
              make_uint4(__half_as_ushort(s0), 0u, 0u, 0u);
        else
          ascale[(size_t)row0 * G + kc] = s0;
      }
    }
    if (v1) {
      if constexpr (MMA_FORM) {
        uint4 o;
        unpack8_e4m3(lo1, o.x, o.y);
        unpack8_e4m3(hi1, o.z, o.w);
        *reinterpret_cast<uint4*>(codes + (size_t)row1 * K + k0) = o;
      } else {
        *reinterpret_cast<uint2*>(codes + (size_t)row1 * (K / 2) + k0 / 2) = make_uint2(lo1, hi1);
      }
      if (c == 0) {
        if constexpr (MMA_FORM)
          *reinterpret_cast<uint4*>(ascale + ((size_t)kc * M + row1) * 8) =
              make_uint4(__half_as_ushort(s1), 0u, 0u, 0u);
        else
          ascale[(size_t)row1 * G + kc] = s1;
      }
    }
    if constexpr (NB > 0) {
      // k is permuted consistently in A and B: logical fragment positions
      // (2c,2c+1 | 2c+8,2c+9) of k16-step s map to physical 16c+4s+(0,1 | 2,3).
#pragma unroll
      for (int j = 0; j < NB; ++j) {
        const uint4* dp = reinterpret_cast<const uint4*>(down_t + (size_t)(8 * j + g) * K + k0);
        uint4 d0 = __ldg(dp), d1 = __ldg(dp + 1);
        uint32_t dw[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          uint32_t a[4] = {w0[2 * s], w1[2 * s], w0[2 * s + 1], w1[2 * s + 1]};
          mma_bf16_16816(acc[j], a, dw[2 * s], dw[2 * s + 1]);
        }
      }
    }
  }

  if constexpr (NB > 0) {
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      red[warp][g][8 * j + 2 * c] = acc[j][0];
      red[warp][g][8 * j + 2 * c + 1] = acc[j][1];
      red[warp][g + 8][8 * j + 2 * c] = acc[j][2];
      red[warp][g + 8][8 * j + 2 * c + 1] = acc[j][3];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < kActRows * RP; i += blockDim.x) {
      const int r = i / RP, col = i % RP;
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kActWarps; ++w) s += red[w][r][col];
      const int row = blockIdx.x * kActRows + r;
      if (row < M) la[(size_t)row * RP + col] = __float2bfloat16_rn(s);
    }
  }
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

template <bool MMA_FORM>
static int launch_act_int4_t(const void* x, const void* smooth, const void* down_t, void* codes,
                             void* ascale, void* la, int M, int K, int rank_pad, cudaStream_t st) {
  dim3 grid((M + kActRows - 1) / kActRows), block(kActWarps * 32);
  auto X = static_cast<const __nv_bfloat16*>(x);
  auto S = static_cast<const __nv_bfloat16*>(smooth);
  auto D = static_cast<const __nv_bfloat16*>(down_t);
  auto C = static_cast<uint8_t*>(codes);
  auto A = static_cast<__half*>(ascale);
  auto L = static_cast<__nv_bfloat16*>(la);
  switch (rank_pad) {
    case 0: act_int4_kernel<0, MMA_FORM><<<grid, block, 0, st>>>(X, S, D, C, A, L, M, K); break;
    case 16: act_int4_kernel<2, MMA_FORM><<<grid, block, 0, st>>>(X, S, D, C, A, L, M, K); break;
    case 32: act_int4_kernel<4, MMA_FORM><<<grid, block, 0, st>>>(X, S, D, C, A, L, M, K); break;
    case 48: act_int4_kernel<6, MMA_FORM><<<grid, block, 0, st>>>(X, S, D, C, A, L, M, K); break;
    case 64: act_int4_kernel<8, MMA_FORM><<<grid, block, 0, st>>>(X, S, D, C, A, L, M, K); break;
    default: return GWB_E_SHAPE;
  }
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

int launch_act_int4(const void* x, const void* smooth, const void* down_t, void* codes,
                    void* ascale, void* la, int M, int K, int rank_pad, bool mma_form,
                    cudaStream_t st) {
  return mma_form ? launch_act_int4_t<true>(x, smooth, down_t, codes, ascale, la, M, K, rank_pad, st)
                  : launch_act_int4_t<false>(x, smooth, down_t, codes, ascale, la, M, K, rank_pad,
                                             st);
}

// Scale interchange form f16 [R, K/64] -> GEMM scale operand rows
// f16 [K/64, R, 8] (scale at k = 0, zeros at k = 1..7).
__global__ void scale_k8_kernel(const __half* __restrict__ scale, uint4* __restrict__ scale_k8,
                                int R, int G) {
  const int64_t n = (int64_t)R * G;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / G, g = i % G;
    scale_k8[(size_t)g * R + r] = make_uint4(__half_as_ushort(scale[i]), 0u, 0u, 0u);
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

int launch_act_int8(const void* x, void* q, void* scale, int M, int K, cudaStream_t st) {
  const int warps_per_block = 8;
  dim3 grid((M + warps_per_block - 1) / warps_per_block), block(warps_per_block * 32);
  act_int8_kernel<<<grid, block, 0, st>>>(static_cast<const __nv_bfloat16*>(x),
                                          static_cast<int8_t*>(q), static_cast<float*>(scale),
                                          M, K);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

}  // namespace gwb
