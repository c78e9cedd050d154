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
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
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
constexpr int PSTAGES = 4;                 // packed staging ring (TMA destination)
constexpr int USTAGES = 3;                 // unpacked ring (MMA operands)
constexpr int PA_BYTES = kBM * kBK / 2;    // 8 KB packed A
constexpr int PB_BYTES = BN * kBK / 2;     // 8 KB packed B
constexpr int PSTAGE_BYTES = PA_BYTES + PB_BYTES;
constexpr int UA_BYTES = kBM * kBK;        // 16 KB
constexpr int UB_BYTES = BN * kBK;         // 16 KB
constexpr int USTAGE_BYTES = UA_BYTES + UB_BYTES;
constexpr int SSTAGES = 8;                 // weight-scale ring (one k-block = 2 groups each)
constexpr int SSTAGE_BYTES = 2 * BN * 4;   // f32 [2 groups][BN]
constexpr int SMEM_BYTES = USTAGES * USTAGE_BYTES + PSTAGES * PSTAGE_BYTES +
                           SSTAGES * SSTAGE_BYTES + 1024 + 512;
constexpr int TMEM_COLS = 256;             // two s32 group buffers of BN columns
constexpr int UNPACK_THREADS = 64;         // warps 2-3
constexpr int EPI_WARPS = 8;               // warps 4-11
constexpr int EC = BN / 2;                 // columns per epilogue warp
constexpr int THREADS = 128 + 32 * EPI_WARPS;
}  // namespace w4

// 8 packed nibbles -> 8 int8 holding 16*q each: the nibble is moved to the
// high half of its byte, which makes the byte the two's-complement value 16*q
// with no sign extension. Output order is (q0 q2 q4 q6)(q1 q3 q5 q7): the
// same k permutation inside every 8-element block of A and of B, which
// leaves each 64-group dot product unchanged; the MMA then sums 256*v, exact
// in s32, and the 1/256 is folded into the activation scale (a power of two,
// so every product and rounding is unchanged).
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t& o0, uint32_t& o1) {
  o0 = (w << 4) & 0xF0F0F0F0u;
  o1 = w & 0xF0F0F0F0u;
}

// Unpack `rows` rows of 64 packed bytes (row-major, no swizzle) into rows of
// 128 int8 in the SWIZZLE_128B K-major layout. Each thread converts one 16B
// packed chunk into two 16B output chunks per iteration.
__device__ __forceinline__ void unpack_tile(const uint8_t* __restrict__ src, uint8_t* dst,
                                            int rows, int tid) {
  for (int i = tid; i < rows * 4; i += w4::UNPACK_THREADS) {
    const int r = i >> 2, cj = i & 3;
    const uint4 p = *reinterpret_cast<const uint4*>(src + r * 64 + cj * 16);
    uint4 o0, o1;
    unpack8(p.x, o0.x, o0.y);
    unpack8(p.y, o0.z, o0.w);
    unpack8(p.z, o1.x, o1.y);
    unpack8(p.w, o1.z, o1.w);
    *reinterpret_cast<uint4*>(dst + swz128(r, cj * 32)) = o0;
    *reinterpret_cast<uint4*>(dst + swz128(r, cj * 32 + 16)) = o1;
  }
}

__global__ void __launch_bounds__(w4::THREADS, 1)
gemm_w4a4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmLA, const __grid_constant__ CUtensorMap tmUP,
                 const __grid_constant__ CUtensorMap tmWS,
                 const __half* __restrict__ a_scale, const float* __restrict__ w_scale_gn,
                 const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ out,
                 int32_t* __restrict__ partials, int M, int N, int K, int rank_pad, int gelu) {
  using namespace w4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ustage = smem;
  uint8_t* pstage = smem + USTAGES * USTAGE_BYTES;
  uint8_t* sstage = pstage + PSTAGES * PSTAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sstage + SSTAGES * SSTAGE_BYTES);
  uint64_t* p_full = bars;
  uint64_t* p_empty = p_full + PSTAGES;
  uint64_t* u_full = p_empty + PSTAGES;
  uint64_t* u_empty = u_full + USTAGES;
  uint64_t* acc_full = u_empty + USTAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint64_t* s_full = acc_empty + 2;         // [SSTAGES]
  uint64_t* s_empty = s_full + SSTAGES;     // [SSTAGES]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_empty + SSTAGES);
  uint32_t* unpack_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
  const int nk = K / kBK;
  const int G = K / 64;
  const bool dump = partials != nullptr;
  const int has_lr = (!dump && rank_pad > 0) ? 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < PSTAGES; ++i) { mbar_init(&p_full[i], 1); mbar_init(&p_empty[i], 1); }
    for (int i = 0; i < USTAGES; ++i) { mbar_init(&u_full[i], 1); mbar_init(&u_empty[i], 1); }
    for (int i = 0; i < 2; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], EPI_WARPS); }
    for (int i = 0; i < SSTAGES; ++i) { mbar_init(&s_full[i], 1); mbar_init(&s_empty[i], EPI_WARPS); }
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
    // ---------------------------------------------------------------- TMA
    if (has_lr) {
      // low-rank operands go straight into unpacked stage 0 (ring slot 0)
      mbar_arrive_expect_tx(&u_full[0], kBM * 128 + BN * 128);
      tma_load_2d(ustage, &tmLA, &u_full[0], 0, m0);
      tma_load_2d(ustage + UA_BYTES, &tmUP, &u_full[0], 0, n0);
    }
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % PSTAGES;
      if (!mbar_wait(&p_empty[s], ((kb / PSTAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER)) break;
      uint8_t* dst = pstage + s * PSTAGE_BYTES;
      mbar_arrive_expect_tx(&p_full[s], PSTAGE_BYTES);
      tma_load_2d(dst, &tmA, &p_full[s], kb * (kBK / 2), m0);
      tma_load_2d(dst + PA_BYTES, &tmB, &p_full[s], kb * (kBK / 2), n0);
      if (!dump) {
        // this k-block's two groups of weight scales, f32 [2][BN]
        const int ss = kb % SSTAGES;
        if (!mbar_wait(&s_empty[ss], ((kb / SSTAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER)) break;
        mbar_arrive_expect_tx(&s_full[ss], SSTAGE_BYTES);
        tma_load_2d(sstage + ss * SSTAGE_BYTES, &tmWS, &s_full[ss], n0, 2 * kb);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------------------------------------------------------- MMA
    constexpr uint32_t idesc = idesc_i8(kBM, BN);
    constexpr uint32_t idesc_lr = idesc_bf16(kBM, BN);
    bool ok = true;
    if (has_lr) {
      // group slot 0 <- la · proj_upᵀ (f32), into accumulator buffer 0
      if (!mbar_wait(&u_full[0], 0, GWB_ERR_TIMEOUT_MMA)) ok = false;
      if (ok && !mbar_wait(&acc_empty[0], 0, GWB_ERR_TIMEOUT_MMA)) ok = false;
      if (ok) {
        tc_fence_after();
        const uint32_t a_base = smem_u32(ustage), b_base = a_base + UA_BYTES;
        for (int k = 0; k < rank_pad / 16; ++k)
          mma_f16(tmem, sdesc_k128(a_base + 32 * k), sdesc_k128(b_base + 32 * k), idesc_lr,
                  k > 0 ? 1u : 0u);
        mma_commit(&acc_full[0]);
        mma_commit(&u_empty[0]);
      }
    }
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int ui = kb + has_lr;
      const int u = ui % USTAGES;
      if (!mbar_wait(&u_full[u], (ui / USTAGES) & 1, GWB_ERR_TIMEOUT_MMA)) { ok = false; break; }
      tc_fence_after();
      const uint32_t a_base = smem_u32(ustage + u * USTAGE_BYTES);
      const uint32_t b_base = a_base + UA_BYTES;
      for (int gs = 0; gs < 2 && ok; ++gs) {
        const int gi = kb * 2 + gs + has_lr;
        const int b = gi & 1;
        // completion #(gi>>1) of acc_empty[b]: #0 is the epilogue's initial
        // magic-bias fill, #j the drain (+ re-bias) of the buffer's use j-1
        if (!mbar_wait(&acc_empty[b], (gi >> 1) & 1, GWB_ERR_TIMEOUT_MMA)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tmem + b * BN;
        // accumulate onto the magic bias already in TMEM
        mma_i8(d, sdesc_k128(a_base + 64 * gs), sdesc_k128(b_base + 64 * gs), idesc, 1u);
        mma_i8(d, sdesc_k128(a_base + 64 * gs + 32), sdesc_k128(b_base + 64 * gs + 32), idesc, 1u);
        mma_commit(&acc_full[b]);
      }
      mma_commit(&u_empty[u]);
    }
  } else if (warp == 2 || warp == 3) {
    // ---------------------------------------------------------------- unpack
    const int tid = threadIdx.x - 64;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % PSTAGES;
      const int ui = kb + has_lr;
      const int u = ui % USTAGES;
      // one thread waits, the named barrier broadcasts the outcome so both
      // unpack warps always leave the loop together
      if (tid == 0) {
        bool ok = mbar_wait(&p_full[s], (kb / PSTAGES) & 1, GWB_ERR_TIMEOUT_UNPACK);
        ok = ok && mbar_wait(&u_empty[u], ((ui / USTAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_UNPACK);
        *unpack_flag = ok ? 1u : 0u;
      }
      asm volatile("bar.sync 1, 64;" ::: "memory");
      if (*reinterpret_cast<volatile uint32_t*>(unpack_flag) == 0u) break;
      const uint8_t* src = pstage + s * PSTAGE_BYTES;
      uint8_t* dst = ustage + u * USTAGE_BYTES;
      unpack_tile(src, dst, kBM, tid);
      unpack_tile(src + PA_BYTES, dst + UA_BYTES, BN, tid);
      fence_proxy_async_smem();
      asm volatile("bar.sync 1, 64;" ::: "memory");
      if (tid == 0) {
        mbar_arrive(&p_empty[s]);
        mbar_arrive(&u_full[u]);
      }
    }
  } else if (warp >= 4) {
    // ---------------------------------------------------------------- epilogue
    // Each s32 group buffer is pre-filled with the bits of 1.5*2^23
    // (0x4B400000); the MMA accumulates the group sum v onto it, so the word
    // read back is the float 1.5*2^23 + v exactly (|v| <= 64*64 < 2^22) and
    // float(v) costs one subtraction instead of an I2F conversion (I2F runs
    // on the narrow conversion pipe). After draining, the epilogue writes the
    // bias back for the buffer's next use. Eight epilogue warps: warp 4+i
    // reads lane quarter i%4 and column slice (i/4)*EC.
    const int q = warp & 3;                  // TMEM lane quarter = tile rows 32q..
    const int cb = ((warp - 4) >> 2) * EC;   // this warp's column slice
    const int row = m0 + 32 * q + lane;
    const bool rv = row < M;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    constexpr uint32_t kMagic = 0x4B400000u;
    const float kMagicF = 12582912.0f;
    uint32_t bias16[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) bias16[j] = kMagic;
#pragma unroll
    for (int bb = 0; bb < 2; ++bb)
#pragma unroll
      for (int c = 0; c < EC; c += 16) tmem_st16(lane_base + bb * BN + cb + c, bias16);
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) { mbar_arrive(&acc_empty[0]); mbar_arrive(&acc_empty[1]); }

    float2 acc[EC / 2];
#pragma unroll
    for (int j = 0; j < EC / 2; ++j) acc[j] = make_float2(0.f, 0.f);
    const float2 negm = make_float2(-kMagicF, -kMagicF);
    const int total = G + has_lr;
    bool ok = true;
    // the activation scale of the next group is fetched one group ahead
    float sa_next = (rv && !dump) ? __half2float(a_scale[(size_t)row * G]) * (1.0f / 256.0f) : 0.f;
    for (int gi = 0; gi < total; ++gi) {
      const int b = gi & 1;
      if (!mbar_wait(&acc_full[b], (gi >> 1) & 1, GWB_ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      tc_fence_after();
      const uint32_t col0 = lane_base + b * BN + cb;
      if (has_lr && gi == 0) {
        // f32 low-rank product la·proj_upᵀ seeds the accumulator
#pragma unroll
        for (int c = 0; c < EC; c += 16) {
          uint32_t v[16];
          tmem_ld16(col0 + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; j += 2)
            acc[(c + j) / 2] = make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1]));
          tmem_st16(col0 + c, bias16);
        }
      } else if (dump) {
        const int g = gi - has_lr;
#pragma unroll
        for (int c = 0; c < EC; c += 16) {
          uint32_t v[16];
          tmem_ld16(col0 + c, v);
          tmem_wait_ld();
          tmem_st16(col0 + c, bias16);
          if (rv) {
            // the MMA summed 256*v (operands hold 16*q)
            uint4* dp = reinterpret_cast<uint4*>(partials + ((size_t)g * M + row) * N + n0 + cb + c);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              dp[j] = make_uint4((uint32_t)((int32_t)(v[4 * j] - kMagic) >> 8),
                                 (uint32_t)((int32_t)(v[4 * j + 1] - kMagic) >> 8),
                                 (uint32_t)((int32_t)(v[4 * j + 2] - kMagic) >> 8),
                                 (uint32_t)((int32_t)(v[4 * j + 3] - kMagic) >> 8));
          }
        }
      } else {
        const int g = gi - has_lr;
        const float sa = sa_next;
        if (rv && g + 1 < G)
          sa_next = __half2float(a_scale[(size_t)row * G + g + 1]) * (1.0f / 256.0f);
        const float2 sa2 = make_float2(sa, sa);
        const int ss = (g >> 1) % SSTAGES;
        if ((g & 1) == 0 &&
            !mbar_wait(&s_full[ss], ((g >> 1) / SSTAGES) & 1, GWB_ERR_TIMEOUT_EPILOGUE)) {
          ok = false;
          break;
        }
        const float* wsg = reinterpret_cast<const float*>(sstage + ss * SSTAGE_BYTES) + (g & 1) * BN + cb;
        uint32_t v[2][16];
        tmem_ld16(col0, v[0]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < EC / 16; ++c) {
          if (c + 1 < EC / 16) tmem_ld16(col0 + (c + 1) * 16, v[(c + 1) & 1]);
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            const float4 ws = *reinterpret_cast<const float4*>(wsg + c * 16 + j);
            const float2 s01 = __fmul2_rn(sa2, make_float2(ws.x, ws.y));
            const float2 s23 = __fmul2_rn(sa2, make_float2(ws.z, ws.w));
            const float2 f01 = __fadd2_rn(
                make_float2(__uint_as_float(v[c & 1][j]), __uint_as_float(v[c & 1][j + 1])), negm);
            const float2 f23 = __fadd2_rn(
                make_float2(__uint_as_float(v[c & 1][j + 2]), __uint_as_float(v[c & 1][j + 3])),
                negm);
            acc[(c * 16 + j) / 2] = __ffma2_rn(f01, s01, acc[(c * 16 + j) / 2]);
            acc[(c * 16 + j) / 2 + 1] = __ffma2_rn(f23, s23, acc[(c * 16 + j) / 2 + 1]);
          }
          tmem_st16(col0 + c * 16, bias16);
          tmem_wait_ld();
        }
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&acc_empty[b]);
        const int g = gi - has_lr;
        if (!dump && g >= 0 && (g & 1) == 1) mbar_arrive(&s_empty[(g >> 1) % SSTAGES]);
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
  if (a.rank_pad > 0 && (!a.la || !a.up)) return GWB_E_SHAPE;
  if (!al16(a.a_codes) || !al16(a.w_codes) || !al16(a.w_scale_gn) ||
      (a.out && !al16(a.out)) || (a.bias && !al16(a.bias)) || (a.la && !al16(a.la)) ||
      (a.up && !al16(a.up)) || (a.partials && !al16(a.partials)))
    return GWB_E_ALIGN;
  if (!a.partials && !a.out) return GWB_E_SHAPE;
  CUtensorMap tA, tB, tLA, tUP, tWS;
  int rc = make_tmap(&tA, a.a_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K / 2, a.M, kBK / 2,
                     kBM, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  rc = make_tmap(&tB, a.w_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K / 2, a.N, kBK / 2,
                 w4::BN, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  tLA = tA;
  tUP = tB;
  tWS = tA;
  if (!a.partials) {
    rc = make_tmap(&tWS, a.w_scale_gn, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.N, a.K / 64, w4::BN,
                   2, CU_TENSOR_MAP_SWIZZLE_NONE);
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
      tA, tB, tLA, tUP, tWS, static_cast<const __half*>(a.a_scale), a.w_scale_gn,
      static_cast<const __nv_bfloat16*>(a.bias), static_cast<__nv_bfloat16*>(a.out), a.partials,
      a.M, a.N, a.K, a.partials ? 0 : a.rank_pad, a.gelu);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

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
