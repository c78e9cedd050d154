// TMA-fed tcgen05 kind::i8 GEMMs for the SVDQuant hot path.
//
//  * gemm_w8a8_kernel: INT8 per-token x INT8 per-output-channel, one s32
//    accumulation over all of K in TMEM, epilogue = s32 -> f32 * a_scale[m] *
//    w_scale[n] + bias[n] (+ GELU tanh) -> bf16.  Tile 128 x 256 x 128.
//  * gemm_w4a4_kernel: packed INT4 (group 64) operands arrive by TMA into a
//    staging ring, unpack warps sign-extend nibbles to int8 in the 128B-swizzled
//    UMMA layout, each 64-wide K group accumulates in its own TMEM s32 buffer
//    (ping-pong), and the epilogue warps promote it into an f32 register
//    accumulator with a_scale[m,g] * w_scale[n,g]. The low-rank branch
//    la·proj_upᵀ is one kind::f16 MMA chain whose f32 result seeds the
//    accumulator; bias / GELU / bf16 conversion happen before the store.
//    Tile 128 x 128 x 128.
//
// Warp roles (both kernels): warp 0 = TMA producer, warp 1 = TMEM owner + MMA
// issuer, warps 2-3 = INT4 unpack (W4A4 only), warps 4-7 = epilogue
// (warp 4+q reads TMEM lanes 32q..32q+31, i.e. tile rows 32q..32q+31).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include "gwb.h"
#include "ptx.cuh"


#ifdef GWB_TRACE
// Optional pipeline trace (compile with -DGWB_TRACE): CTA (0,0) of the W4A4
// GEMM records clock64() at each role's events; gwb_trace_read copies it out.
__device__ long long gwb_trace[8][512];
#define GWB_TRACE_AT(role, idx) do { if (blockIdx.x == 0 && blockIdx.y == 0 && (idx) < 512) \
    gwb_trace[role][idx] = clock64(); } while (0)
#else
#define GWB_TRACE_AT(role, idx) do { } while (0)
#endif

namespace gwb {

constexpr int kThreads = 256;
constexpr int kBM = 128;
constexpr int kBK = 128;  // int8 elements (= bytes) per k-block: one 128B swizzle row

__device__ __forceinline__ float gelu_tanh(float v) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  return 0.5f * v * (1.0f + tanhf(k0 * (v + k1 * v * v * v)));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ======================================================================
// W8A8
// ======================================================================
namespace w8 {
constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int A_BYTES = kBM * kBK;        // 16 KB
constexpr int B_BYTES = BN * kBK;         // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr int TMEM_COLS = 256;
}  // namespace w8

__global__ void __launch_bounds__(kThreads, 1)
gemm_w8a8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const float* __restrict__ a_scale, const float* __restrict__ w_scale,
                 const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ out,
                 int M, int N, int K, int gelu) {
  using namespace w8;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment by offsetting the __shared__ array itself, so the
  // compiler keeps emitting shared-space (not generic) loads and stores
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
  const int nk = K / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    mbar_init(acc_full, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % STAGES;
      if (!mbar_wait(&empty[s], ((kb / STAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER)) break;
      uint8_t* sa = smem + s * STAGE_BYTES;
      mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
      tma_load_2d(sa, &tmA, &full[s], kb * kBK, m0);
      tma_load_2d(sa + A_BYTES, &tmB, &full[s], kb * kBK, n0);
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = idesc_i8(kBM, BN);
    bool ok = true;
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % STAGES;
      if (!mbar_wait(&full[s], (kb / STAGES) & 1, GWB_ERR_TIMEOUT_MMA)) { ok = false; break; }
      tc_fence_after();
      const uint32_t a_base = smem_u32(smem + s * STAGE_BYTES);
      const uint32_t b_base = a_base + A_BYTES;
#pragma unroll
      for (int k = 0; k < kBK / 32; ++k) {
        mma_i8(tmem, sdesc_k128(a_base + 32 * k), sdesc_k128(b_base + 32 * k), idesc,
               (kb > 0 || k > 0) ? 1u : 0u);
      }
      mma_commit(&empty[s]);
    }
    if (ok) mma_commit(acc_full);
  } else if (warp >= 4) {
    const int q = warp - 4;
    const int row = m0 + 32 * q + lane;
    if (mbar_wait(acc_full, 0, GWB_ERR_TIMEOUT_EPILOGUE)) {
      tc_fence_after();
      const float sa = row < M ? a_scale[row] : 0.f;
      for (int c = 0; c < BN; c += 16) {
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + c, v);
        tmem_wait_ld();
        if (row < M) {
          float f[16];
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            const float4 ws = *reinterpret_cast<const float4*>(w_scale + n0 + c + j);
            f[j + 0] = (float)(int)v[j + 0] * sa * ws.x;
            f[j + 1] = (float)(int)v[j + 1] * sa * ws.y;
            f[j + 2] = (float)(int)v[j + 2] * sa * ws.z;
            f[j + 3] = (float)(int)v[j + 3] * sa * ws.w;
          }
          if (bias != nullptr) {
            const uint4* bp = reinterpret_cast<const uint4*>(bias + n0 + c);
            uint4 b0 = __ldg(bp), b1 = __ldg(bp + 1);
            uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              f[2 * j] += __uint_as_float(bw[j] << 16);
              f[2 * j + 1] += __uint_as_float(bw[j] & 0xFFFF0000u);
            }
          }
          if (gelu) {
#pragma unroll
            for (int j = 0; j < 16; ++j) f[j] = gelu_tanh(f[j]);
          }
          uint4* op = reinterpret_cast<uint4*>(out + (size_t)row * N + n0 + c);
          op[0] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                             pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
          op[1] = make_uint4(pack_bf16x2(f[8], f[9]), pack_bf16x2(f[10], f[11]),
                             pack_bf16x2(f[12], f[13]), pack_bf16x2(f[14], f[15]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ======================================================================
// W4A4 (INT4 group-64, unpacked to int8 in shared memory)
// ======================================================================
namespace w4 {
constexpr int BN = 128;
constexpr int STAGES = 4;                  // operand ring (all TMA-fed)
constexpr int A_BYTES = kBM * kBK;         // 16 KB e4m3 A (activation operand form)
constexpr int B_BYTES = BN * kBK;          // 16 KB e4m3 B (expanded weight)
// Scale operand of one group and side: [128 rows x 16 k] f16, no-swizzle
// K-major. TMA writes the k = 0..7 half (one 16-byte row per matrix row, only
// k = 0 non-zero); the k = 8..15 half is a 2 KB zero block LBO = 2 KB away.
constexpr int SOP_DATA = 128 * 16;         // 2 KB
constexpr int SOP_BYTES = 2 * SOP_DATA;    // 4 KB incl. the zero half
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + 4 * SOP_BYTES;   // 48 KB
constexpr int TX_BYTES = A_BYTES + B_BYTES + 4 * SOP_DATA;       // 40 KB by TMA
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
// TMEM: [0, 2*BN) f32 group sums V0/V1, [2*BN, 4*BN) f32 scale products S0/S1
constexpr int TMEM_COLS = 512;
constexpr int EPI_WARPS = 8;               // warps 4-11 (warpgroups 1-2)
constexpr int EC = BN / 2;                 // columns per epilogue warp
constexpr int THREADS = 128 + 32 * EPI_WARPS;   // warps 2-3 idle: warpgroup 0 padding
}  // namespace w4

static_assert(w4::SMEM_BYTES <= 232448, "W4A4 shared memory exceeds 227 KB");

// Shared-memory descriptor of a scale operand: K-major, no swizzle, 8-row x
// 16-byte core matrices stored contiguously (SBO = 128 B between 8-row
// blocks), the k = 8..15 half LBO = 2 KB away (layout type 0).
__device__ __forceinline__ uint64_t sdesc_scale(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)(w4::SOP_DATA >> 4) << 16;
  d |= (uint64_t)(128u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

__global__ void __launch_bounds__(w4::THREADS, 1)
gemm_w4a4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmAS, const __grid_constant__ CUtensorMap tmBS,
                 const __grid_constant__ CUtensorMap tmLA, const __grid_constant__ CUtensorMap tmUP,
                 const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ out,
                 int32_t* __restrict__ partials, int M, int N, int K, int rank_pad, int gelu) {
  using namespace w4;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment by offsetting the __shared__ array itself, so the
  // compiler keeps emitting shared-space (not generic) loads and stores
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;                    // [STAGES]
  uint64_t* empty = full + STAGES;          // [STAGES]
  uint64_t* acc_full = empty + STAGES;      // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
  const int nk = K / kBK;
  const int G = K / 64;
  const bool dump = partials != nullptr;
  const int has_lr = (!dump && rank_pad > 0) ? 1 : 0;

  // zero halves of the scale operands (never written by TMA)
  for (int st = 0; st < STAGES; ++st)
    for (int o = 0; o < 4; ++o) {
      uint4* z = reinterpret_cast<uint4*>(smem + st * STAGE_BYTES + A_BYTES + B_BYTES +
                                          o * SOP_BYTES + SOP_DATA);
      for (int i = threadIdx.x; i < SOP_DATA / 16; i += THREADS) z[i] = make_uint4(0, 0, 0, 0);
    }
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], EPI_WARPS); }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmAS);
    tma_prefetch_desc(&tmBS);
  }
  if (warp == 1) { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) GWB_TRACE_AT(7, 0);
  // register hand-off: the launch gives 384 x 168 = 64512 registers;
  // warpgroup 0 (producer, MMA, two idle warps) drops to 40 (5120) and the
  // two epilogue warpgroups rise to 232 (59392): 64512 in total
  if (warp < 4) {
  regs_dec<40>();
  if (warp == 0 && lane == 0) {
    // ---------------------------------------------------------------- TMA
    if (has_lr) {
      // low-rank operands go straight into stage 0 (ring slot 0)
      mbar_arrive_expect_tx(&full[0], kBM * 128 + BN * 128);
      tma_load_2d(smem, &tmLA, &full[0], 0, m0);
      tma_load_2d(smem + A_BYTES, &tmUP, &full[0], 0, n0);
    }
    for (int kb = 0; kb < nk; ++kb) {
      const int ui = kb + has_lr, s = ui % STAGES;
      if (!mbar_wait(&empty[s], ((ui / STAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER)) break;
      GWB_TRACE_AT(0, kb);
      uint8_t* st = smem + s * STAGE_BYTES;
      mbar_arrive_expect_tx(&full[s], dump ? A_BYTES + B_BYTES : TX_BYTES);
      tma_load_2d(st, &tmA, &full[s], kb * kBK, m0);
      tma_load_2d(st + A_BYTES, &tmB, &full[s], kb * kBK, n0);
      if (!dump) {
        uint8_t* so = st + A_BYTES + B_BYTES;
#pragma unroll
        for (int gs = 0; gs < 2; ++gs) {
          const int g = 2 * kb + gs;
          tma_load_2d(so + (2 * gs) * SOP_BYTES, &tmAS, &full[s], 0, g * M + m0);
          tma_load_2d(so + (2 * gs + 1) * SOP_BYTES, &tmBS, &full[s], 0, g * N + n0);
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA
    constexpr uint32_t idesc = idesc_fmt0_f32(kBM, BN);      // e4m3 x e4m3 -> f32
    constexpr uint32_t idesc_lr = idesc_bf16(kBM, BN);
    constexpr uint32_t idesc_s = idesc_fmt0_f32(kBM, BN);    // f16 x f16 -> f32
    bool ok = true;
    if (has_lr) {
      // group slot 0 <- la · proj_upᵀ (f32), into accumulator buffer 0
      if (!mbar_wait(&full[0], 0, GWB_ERR_TIMEOUT_MMA)) ok = false;
      if (ok && !mbar_wait(&acc_empty[0], 1, GWB_ERR_TIMEOUT_MMA)) ok = false;
      if (ok) {
        tc_fence_after();
        const uint32_t a_base = smem_u32(smem), b_base = a_base + A_BYTES;
        for (int k = 0; k < rank_pad / 16; ++k)
          mma_f16(tmem, sdesc_k128(a_base + 32 * k), sdesc_k128(b_base + 32 * k), idesc_lr,
                  k > 0 ? 1u : 0u);
        mma_commit(&acc_full[0]);
        mma_commit(&empty[0]);
      }
    }
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int ui = kb + has_lr, s = ui % STAGES;
      if (!mbar_wait(&full[s], (ui / STAGES) & 1, GWB_ERR_TIMEOUT_MMA)) { ok = false; break; }
      GWB_TRACE_AT(1, kb);
      tc_fence_after();
      const uint32_t a_base = smem_u32(smem + s * STAGE_BYTES);
      const uint32_t b_base = a_base + A_BYTES;
      const uint32_t s_base = b_base + B_BYTES;
      for (int gs = 0; gs < 2 && ok; ++gs) {
        const int gi = kb * 2 + gs + has_lr;
        const int b = gi & 1;
        if (!mbar_wait(&acc_empty[b], ((gi >> 1) & 1) ^ 1, GWB_ERR_TIMEOUT_MMA)) { ok = false; break; }
        GWB_TRACE_AT(2, gi);
        tc_fence_after();
        const uint32_t d = tmem + b * BN;
        mma_f8(d, sdesc_k128(a_base + 64 * gs), sdesc_k128(b_base + 64 * gs), idesc, 0u);
        mma_f8(d, sdesc_k128(a_base + 64 * gs + 32), sdesc_k128(b_base + 64 * gs + 32), idesc, 1u);
        if (!dump) {
          // S_b = a_scale[:, g] ⊗ w_scale[:, g], exact in f32 (11-bit x 11-bit)
          const uint32_t so = s_base + 2 * gs * SOP_BYTES;
          mma_f16(tmem + 2 * BN + b * BN, sdesc_scale(so), sdesc_scale(so + SOP_BYTES), idesc_s,
                  0u);
        }
        mma_commit(&acc_full[b]);
      }
      mma_commit(&empty[s]);
    }
  }
  } else {
    regs_inc<232>();
    // ---------------------------------------------------------------- epilogue
    // Per group: load the f32 group sum V (an exact integer: e4m3 operands
    // hold the INT4 codes themselves) of this warp's 32 rows x EC columns and
    // the scale product S = a_scale * w_scale the tensor core wrote beside it,
    // wait once, hand the TMEM buffer straight back to the MMA warp, then
    // acc += V * S (one FFMA per element). Warps 4..11: lane quarter warp % 4
    // (tile rows 32*(warp%4)..), column slice ((warp-4)/4)*EC.
    const int q = warp & 3;
    const int cb = ((warp - 4) >> 2) * EC;
    const int row = m0 + 32 * q + lane;
    const bool rv = row < M;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    float2 acc[EC / 2];
#pragma unroll
    for (int j = 0; j < EC / 2; ++j) acc[j] = make_float2(0.f, 0.f);
    const int total = G + has_lr;
    bool ok = true;
    for (int gi = 0; gi < total; ++gi) {
      const int b = gi & 1;
      if (!mbar_wait(&acc_full[b], (gi >> 1) & 1, GWB_ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      if (warp == 4 && lane == 0) GWB_TRACE_AT(5, gi);
      tc_fence_after();
      const uint32_t col0 = lane_base + b * BN + cb;
      const bool lr = has_lr && gi == 0;
      uint32_t v[EC], sc[EC];
#pragma unroll
      for (int c = 0; c < EC; c += 32) tmem_ld32(col0 + c, v + c);
      if (!lr && !dump) {
#pragma unroll
        for (int c = 0; c < EC; c += 32) tmem_ld32(col0 + 2 * BN + c, sc + c);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (warp == 4 && lane == 0) GWB_TRACE_AT(6, gi);
      if (lr) {
        // f32 low-rank product la·proj_upᵀ seeds the accumulator
#pragma unroll
        for (int j = 0; j < EC; j += 2)
          acc[j / 2] = make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1]));
      } else if (dump) {
        if (rv) {
          const int g = gi - has_lr;
          uint4* dp = reinterpret_cast<uint4*>(partials + ((size_t)g * M + row) * N + n0 + cb);
#pragma unroll
          for (int j = 0; j < EC / 4; ++j)
            dp[j] = make_uint4((uint32_t)__float2int_rn(__uint_as_float(v[4 * j])),
                               (uint32_t)__float2int_rn(__uint_as_float(v[4 * j + 1])),
                               (uint32_t)__float2int_rn(__uint_as_float(v[4 * j + 2])),
                               (uint32_t)__float2int_rn(__uint_as_float(v[4 * j + 3])));
        }
      } else {
#pragma unroll
        for (int j = 0; j < EC; j += 2)
          acc[j / 2] = __ffma2_rn(make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])),
                                  make_float2(__uint_as_float(sc[j]), __uint_as_float(sc[j + 1])),
                                  acc[j / 2]);
      }
    }
    if (ok && !dump && rv) {
#pragma unroll
      for (int c = 0; c < EC; c += 8) {
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; j += 2) {
          f[j] = acc[(c + j) / 2].x;
          f[j + 1] = acc[(c + j) / 2].y;
        }
        if (bias != nullptr) {
          const uint4 bw = __ldg(reinterpret_cast<const uint4*>(bias + n0 + cb + c));
          const uint32_t w[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            f[2 * j] += __uint_as_float(w[j] << 16);
            f[2 * j + 1] += __uint_as_float(w[j] & 0xFFFF0000u);
          }
        }
        if (gelu) {
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] = gelu_tanh(f[j]);
        }
        *reinterpret_cast<uint4*>(out + (size_t)row * N + n0 + cb + c) =
            make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                       pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ======================================================================
// host side: tensor maps + launches
// ======================================================================
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D row-major tensor [rows][cols] of `esize`-byte elements; box = {bx, by}.
static int make_tmap(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int esize,
                     uint64_t cols, uint64_t rows, uint32_t bx, uint32_t by,
                     CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return GWB_E_DRIVER;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * (uint64_t)esize};
  cuuint32_t box[2] = {bx, by};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? GWB_SUCCESS : GWB_E_TMAP;
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_gemm_w8a8(const W8A8Args& a, cudaStream_t st) {
  if (a.M <= 0 || a.K <= 0 || a.K % kBK || a.N % w8::BN) return GWB_E_SHAPE;
  if (!al16(a.a_q) || !al16(a.w_q) || !al16(a.out) || !al16(a.w_scale) ||
      (a.bias && !al16(a.bias)))
    return GWB_E_ALIGN;
  CUtensorMap tA, tB;
  int rc = make_tmap(&tA, a.a_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K, a.M, kBK, kBM,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap(&tB, a.w_q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K, a.N, kBK, w8::BN,
                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemm_w8a8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         w8::SMEM_BYTES);
    attr = true;
  }
  dim3 grid(a.N / w8::BN, (a.M + kBM - 1) / kBM);
  gemm_w8a8_kernel<<<grid, kThreads, w8::SMEM_BYTES, st>>>(
      tA, tB, a.a_scale, a.w_scale, static_cast<const __nv_bfloat16*>(a.bias),
      static_cast<__nv_bfloat16*>(a.out), a.M, a.N, a.K, a.gelu);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

int launch_gemm_w4a4(const W4A4Args& a, cudaStream_t st) {
  if (a.M <= 0 || a.K <= 0 || a.K % kBK || a.N % w4::BN) return GWB_E_SHAPE;
  if (a.rank_pad < 0 || a.rank_pad > 64 || a.rank_pad % 16) return GWB_E_SHAPE;
  if (a.rank_pad > 0 && !a.partials && (!a.la || !a.up)) return GWB_E_SHAPE;
  if (!a.partials && !a.out) return GWB_E_SHAPE;
  const int G = a.K / 64;
  if ((int64_t)G * a.M > 0x7fffffff || (int64_t)G * a.N > 0x7fffffff) return GWB_E_SHAPE;
  if (!al16(a.a_q8) || !al16(a.w_q8) || (a.out && !al16(a.out)) || (a.bias && !al16(a.bias)) ||
      (a.la && !al16(a.la)) || (a.up && !al16(a.up)) || (a.partials && !al16(a.partials)) ||
      (!a.partials && (!al16(a.a_scale_k8) || !al16(a.w_scale_k8))))
    return GWB_E_ALIGN;
  CUtensorMap tA, tB, tAS, tBS, tLA, tUP;
  int rc = make_tmap(&tA, a.a_q8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K, a.M, kBK, kBM,
                     CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap(&tB, a.w_q8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K, a.N, kBK, w4::BN,
                 CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  tAS = tA;
  tBS = tB;
  tLA = tA;
  tUP = tB;
  if (!a.partials) {
    rc = make_tmap(&tAS, a.a_scale_k8, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 8, (uint64_t)G * a.M,
                   8, kBM, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = make_tmap(&tBS, a.w_scale_k8, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 8, (uint64_t)G * a.N,
                   8, w4::BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  if (a.rank_pad > 0 && !a.partials) {
    rc = make_tmap(&tLA, a.la, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.rank_pad, a.M, 64, kBM,
                   CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap(&tUP, a.up, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.rank_pad, a.N, 64, w4::BN,
                   CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemm_w4a4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         w4::SMEM_BYTES);
    attr = true;
  }
  dim3 grid(a.N / w4::BN, (a.M + kBM - 1) / kBM);
  gemm_w4a4_kernel<<<grid, w4::THREADS, w4::SMEM_BYTES, st>>>(
      tA, tB, tAS, tBS, tLA, tUP, static_cast<const __nv_bfloat16*>(a.bias),
      static_cast<__nv_bfloat16*>(a.out), a.partials, a.M, a.N, a.K,
      a.partials ? 0 : a.rank_pad, a.gelu);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

#ifdef GWB_TRACE
}  // namespace gwb
extern "C" int gwb_trace_read(long long* dst) {
  return cudaMemcpyFromSymbol(dst, gwb_trace, sizeof(long long) * 8 * 512) == cudaSuccess ? 0 : 3;
}
namespace gwb {
#endif

int device_error_read_and_clear(int* code) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gwb_dev_error, sizeof(int)) != cudaSuccess) return GWB_E_LAUNCH;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(gwb_dev_error, &zero, sizeof(int));
  }
  *code = v;
  return GWB_SUCCESS;
}

}  // namespace gwb
