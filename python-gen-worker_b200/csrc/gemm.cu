// TMA-fed tcgen05 GEMMs for the SVDQuant hot path (persistent tiles).
//
//  * gemm_w8a8_kernel: W8A8 per-token x per-output-channel, INT8 (kind::i8,
//    s32 accumulator) or FP8 e4m3 (kind::f8f6f4, f32 accumulator); one
//    accumulation over all of K in TMEM (two accumulators, so one tile's
//    epilogue overlaps the next tile's k-loop); epilogue = acc * a_scale[m] *
//    w_scale[n] + bias[n] (+ GELU tanh) -> bf16. Tile 128 x 256 x 128.
//  * gemm_w4a4_kernel: INT4 group-64 codes as e4m3 operands (q * 2^-9): per
//    64-group the tensor core forms the exact group sum V (f32, TMEM) and the
//    scale product S = a_scale ⊗ w_scale (kind::f16, TMEM); the epilogue
//    promotes acc += V * S in registers. The low-rank branch la·proj_upᵀ is
//    one kind::f16 MMA chain whose f32 result seeds the accumulator; bias /
//    GELU / bf16 conversion happen before the store. Activations arrive in
//    the operand form or as packed codes expanded in shared memory.
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

constexpr int kBM = 128;
constexpr int kBK = 128;  // int8 elements (= bytes) per k-block: one 128B swizzle row

// GELU, tanh form: 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3))). tanh is
// the hardware approximation (tanh.approx.f32, |error| < 2^-10.9), far below
// the bf16 rounding of the output.
__device__ __forceinline__ float gelu_tanh(float v) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  const float k1 = 0.044715f;
  const float u = k0 * (v + k1 * v * v * v);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * v * (1.0f + t);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ======================================================================
// W8A8
// ======================================================================
// Persistent: each CTA walks tiles blockIdx.x, +gridDim.x, ... The two TMEM
// accumulators (2 x 256 columns) let the MMA run tile i+1's k-loop while the
// epilogue warps drain tile i, so the epilogue (scales, bias, GELU, store)
// is hidden behind the tensor core instead of following it.
namespace w8 {
constexpr int BN = 256;
constexpr int STAGES = 4;
constexpr int A_BYTES = kBM * kBK;        // 16 KB
constexpr int B_BYTES = BN * kBK;         // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NACC = 2;                   // TMEM accumulators (tile ping-pong)
constexpr int TMEM_COLS = NACC * BN;      // 512
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
// 12 warps: 0 TMA, 1 MMA, 2-3 idle, 4-11 epilogue (lane quarter warp % 4,
// column half ((warp - 4) / 4) * EC).
constexpr int THREADS = 384;
constexpr int EPI0 = 4;
constexpr int EPI_WARPS = 8;
constexpr int EC = BN / 2;
}  // namespace w8

// FP8 = false: s8 x s8 -> s32 (kind::i8); FP8 = true: e4m3 x e4m3 -> f32
// (kind::f8f6f4), the reference's own W8A8 number format.
template <bool FP8>
__global__ void __launch_bounds__(w8::THREADS, 1)
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
  uint64_t* acc_full = empty + STAGES;      // [NACC]
  uint64_t* acc_empty = acc_full + NACC;    // [NACC]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + NACC);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = K / kBK;
  const int tiles_n = N / BN;
  const int ntiles = ((M + kBM - 1) / kBM) * tiles_n;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 1); }
    for (int i = 0; i < NACC; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], EPI_WARPS); }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // register hand-off: 384 x 168 = 64512 at launch; warpgroup 0 drops to 40
  // (5120), the two epilogue warpgroups rise to 232 (59392)
  if (warp < EPI0) {
    regs_dec<40>();
    if (warp == 0 && lane == 0) {
      // -------------------------------------------------------------- TMA
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        const int m0 = (tile / tiles_n) * kBM, n0 = (tile % tiles_n) * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * STAGE_BYTES;
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(sa, &tmA, &full[s], kb * kBK, m0);
          tma_load_2d(sa + A_BYTES, &tmB, &full[s], kb * kBK, n0);
        }
      }
    } else if (warp == 1 && lane == 0) {
      // -------------------------------------------------------------- MMA
      constexpr uint32_t idesc = FP8 ? idesc_fmt0_f32(kBM, BN) : idesc_i8(kBM, BN);
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++lt) {
        const int b = lt & 1;
        if (!mbar_wait(&acc_empty[b], ((lt >> 1) & 1) ^ 1, GWB_ERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d = tmem + b * BN;
        for (int kb = 0; kb < nk; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(&full[s], (it / STAGES) & 1, GWB_ERR_TIMEOUT_MMA)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t b_base = a_base + A_BYTES;
#pragma unroll
          for (int k = 0; k < kBK / 32; ++k) {
            if constexpr (FP8)
              mma_f8(d, sdesc_k128(a_base + 32 * k), sdesc_k128(b_base + 32 * k), idesc,
                     (kb > 0 || k > 0) ? 1u : 0u);
            else
              mma_i8(d, sdesc_k128(a_base + 32 * k), sdesc_k128(b_base + 32 * k), idesc,
                     (kb > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&acc_full[b]);
      }
    }
  } else {
    regs_inc<232>();
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int cb = ((warp - EPI0) >> 2) * EC;
    int lt = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++lt) {
      const int m0 = (tile / tiles_n) * kBM, n0 = (tile % tiles_n) * BN;
      const int b = lt & 1;
      if (!mbar_wait(&acc_full[b], (lt >> 1) & 1, GWB_ERR_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      // the whole 32-row x 128-column slice goes to registers, then the
      // accumulator is handed back before any arithmetic
      uint32_t v[EC];
      const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) + b * BN + cb;
#pragma unroll
      for (int c = 0; c < EC; c += 32) tmem_ld32(base + c, v + c);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      const int row = m0 + 32 * q + lane;
      if (row >= M) continue;
      const float sa = a_scale[row];
      uint4* op = reinterpret_cast<uint4*>(out + (size_t)row * N + n0 + cb);
#pragma unroll
      for (int c = 0; c < EC; c += 8) {
        const float4 w0 = __ldg(reinterpret_cast<const float4*>(w_scale + n0 + cb + c));
        const float4 w1 = __ldg(reinterpret_cast<const float4*>(w_scale + n0 + cb + c + 4));
        const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
          f[j] = (FP8 ? __uint_as_float(v[c + j]) : (float)(int)v[c + j]) * sa * ws[j];
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
        op[c / 8] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                               pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
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
constexpr int PSTAGES = 4;                 // packed-code staging ring (TMA)
constexpr int UA_BYTES = kBM * kBK;        // 16 KB e4m3 A (unpacked here)
// Scale operand of one group and side: [rows x 16 k] f16, no-swizzle
// K-major. TMA writes the k = 0..7 half (one 16-byte row per matrix row: the
// A side one-hot at k = g mod 8, the B side one-hot alike or the stored 8
// groups g - g mod 8 .. +7); the k = 8..15 half is the shared 2 KB zero block.
constexpr int SOPA = kBM * 16;             // 2 KB (A side, 128 rows)
constexpr int ZERO_BYTES = SOPA;
constexpr int TMEM_COLS = 512;
// unpack warps from warp 2 on: six (warps 2-7) when the activations arrive
// packed, else two (warps 2-3, the warpgroup's otherwise idle pair) for a
// packed weight alone
template <bool A_PACKED> __host__ __device__ constexpr int unpack_threads() {
  return A_PACKED ? 192 : 64;
}
constexpr int EPI_WARPS = 8;               // the last two warpgroups
// Tile N width BN: 128 (two TMEM group buffers of V | S) or 64 (four).
// TMEM: [0, NBUF*BN) f32 group sums V_b, [NBUF*BN, 512) f32 scale products S_b.
template <bool A_PACKED, bool B_PACKED, int BN> struct Cfg {
  static constexpr int NBUF = TMEM_COLS / (2 * BN);
  static constexpr int UB_BYTES = BN * kBK;                 // e4m3 B
  static constexpr int SOPB = BN * 16;                      // one B scale-operand tile
  // per k-block scale operands: two A one-hot tiles, then one stored 8-group
  // B tile (B_PACKED) or two B one-hot tiles
  static constexpr int SCALE_BYTES = 2 * SOPA + (B_PACKED ? 1 : 2) * SOPB;
  static constexpr int USTAGE_BYTES = UA_BYTES + UB_BYTES + SCALE_BYTES;
  static constexpr int PA_STAGE = A_PACKED ? kBM * kBK / 2 : 0;   // packed A per k-block
  static constexpr int PB_STAGE = B_PACKED ? BN * kBK / 2 : 0;    // packed B per k-block
  static constexpr int FIXED = PSTAGES * (PA_STAGE + PB_STAGE) + ZERO_BYTES + 1024 + 256;
  static constexpr int FIT = (232448 - FIXED) / USTAGE_BYTES;      // operand stages that fit
  static constexpr int USTAGES = FIT < 6 ? FIT : 6;               // operand ring read by the MMA
  static constexpr int ZERO_OFF = USTAGES * USTAGE_BYTES + PSTAGES * (PA_STAGE + PB_STAGE);
  static constexpr int SMEM_BYTES = ZERO_OFF + ZERO_BYTES + 1024 + 256;
  static constexpr int EC = BN / 2;                         // columns per epilogue warp
  static_assert(USTAGES >= 3, "W4A4 operand ring too small");
  static_assert(SMEM_BYTES <= 232448, "W4A4 shared memory exceeds 227 KB");
};
// packed activations: 16 warps (producer, MMA, 6 unpack, 8 epilogue);
// operand-form activations: 12 warps (producer, MMA, 2 unpack or idle, 8 epilogue)
template <bool A_PACKED> __host__ __device__ constexpr int threads() { return A_PACKED ? 512 : 384; }
template <bool A_PACKED> __host__ __device__ constexpr int epi_warp0() { return A_PACKED ? 8 : 4; }
// Both operands hold q * 2^-9 (e4m3 subnormals), so a group sum is
// 2^-18 * v exactly; the accumulator is kept in that scale and multiplied by
// 2^18 (exact) once at the end of the tile.
constexpr float kUnscale = 262144.0f;      // 2^18
constexpr float kRescale = 1.0f / 262144.0f;
}  // namespace w4


// Unpack `chunks` 16-byte packed chunks (rows of 64 packed bytes, row-major,
// no swizzle) into rows of 128 e4m3 bytes in the SWIZZLE_128B K-major layout.
template <int kRows, int kThreads>
__device__ __forceinline__ void unpack_tile(const uint8_t* __restrict__ src, uint8_t* dst,
                                            int tid) {
  constexpr int kChunks = kRows * 4;
  constexpr int kPer = (kChunks + kThreads - 1) / kThreads;
  constexpr int kBatch = kPer < 4 ? kPer : 4;   // loads in flight per thread
#pragma unroll
  for (int j0 = 0; j0 < kPer; j0 += kBatch) {
  uint4 p[kBatch];
#pragma unroll
  for (int jj = 0; jj < kBatch; ++jj) {
    const int i = tid + (j0 + jj) * kThreads;
    if (j0 + jj < kPer && i < kChunks)
      p[jj] = *reinterpret_cast<const uint4*>(src + (i >> 2) * 64 + (i & 3) * 16);
  }
#pragma unroll
  for (int jj = 0; jj < kBatch; ++jj) {
    const int j = jj;
    const int i = tid + (j0 + jj) * kThreads;
    if (j0 + jj < kPer && i < kChunks) {
      const int r = i >> 2, cj = i & 3;
      uint4 o0, o1;
      unpack8_e4m3(p[j].x, o0.x, o0.y);
      unpack8_e4m3(p[j].y, o0.z, o0.w);
      unpack8_e4m3(p[j].z, o1.x, o1.y);
      unpack8_e4m3(p[j].w, o1.z, o1.w);
      *reinterpret_cast<uint4*>(dst + swz128(r, cj * 32)) = o0;
      *reinterpret_cast<uint4*>(dst + swz128(r, cj * 32 + 16)) = o1;
    }
  }
}
}

// Load-time weight expansion: packed sign-magnitude nibbles u8 [N, K/2] ->
// e4m3 bytes q * 2^-9 u8 [N, K] in the operand order of unpack8_e4m3, so the
// weight tile is TMA-loaded straight into the MMA operand layout.
__global__ void w4a4_weight_expand_kernel(const uint32_t* __restrict__ packed,
                                          uint2* __restrict__ out, int64_t nwords) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nwords;
       i += (int64_t)gridDim.x * blockDim.x) {
    uint2 o;
    unpack8_e4m3(packed[i], o.x, o.y);
    out[i] = o;
  }
}

// Shared-memory descriptor of a scale operand: K-major, no swizzle, 8-row x
// 16-byte core matrices stored contiguously (SBO = 128 B between 8-row
// blocks); the k = 8..15 half is the shared zero block, `lbo` bytes away
// (layout type 0).
__device__ __forceinline__ uint64_t sdesc_scale(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(128u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// A_PACKED: activations arrive as packed INT4 codes (TMA into the staging
// ring, expanded to the operand layout by the unpack warps); otherwise as the
// operand form itself (u8 [M, K], TMA straight into the operand ring).
// B_PACKED: the weight arrives as stored, packed INT4 codes u8 [N, K/2]
// (expanded in shared memory by the unpack warps) with its group scales as
// stored, f16 [N, G]: TMA brings 8 groups per row (16 bytes, the no-swizzle
// K-major core-matrix layout) and that tile is the B side of the scale MMA
// of both groups of the k-block; the A side (one-hot at k = g mod 8, written
// by the quantiser) selects the group. Otherwise the weight is the load-time
// operand form (w_q8 u8 [N, K], w_scale_k8 one-hot rows).
template <bool A_PACKED, bool B_PACKED, int BN>
__global__ void __launch_bounds__(w4::threads<A_PACKED>(), 1)
gemm_w4a4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmAS, const __grid_constant__ CUtensorMap tmBS,
                 const __grid_constant__ CUtensorMap tmLA, const __grid_constant__ CUtensorMap tmUP,
                 const __nv_bfloat16* __restrict__ bias, __nv_bfloat16* __restrict__ out,
                 int32_t* __restrict__ partials, int M, int N, int K, int rank_pad, int gelu) {
  using namespace w4;
  using C = Cfg<A_PACKED, B_PACKED, BN>;
  constexpr bool UNPACK = A_PACKED || B_PACKED;
  constexpr int NBUF = C::NBUF, USTAGES = C::USTAGES, USTAGE_BYTES = C::USTAGE_BYTES;
  constexpr int UB_BYTES = C::UB_BYTES, SOPB = C::SOPB, SCALE_BYTES = C::SCALE_BYTES;
  constexpr int PA = C::PA_STAGE, PB = C::PB_STAGE;
  constexpr int EC = C::EC;
  constexpr int THREADS = threads<A_PACKED>();
  constexpr int EPI0 = epi_warp0<A_PACKED>();
  constexpr int UNPACK_THREADS = unpack_threads<A_PACKED>();
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment by offsetting the __shared__ array itself, so the
  // compiler keeps emitting shared-space (not generic) loads and stores
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* ustage = smem;
  uint8_t* pstage = smem + USTAGES * USTAGE_BYTES;
  uint8_t* zero = smem + C::ZERO_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(zero + ZERO_BYTES);
  uint64_t* p_full = bars;                  // [PSTAGES] packed codes landed (TMA)
  uint64_t* p_empty = p_full + PSTAGES;     // [PSTAGES] unpack done reading
  uint64_t* u_full = p_empty + PSTAGES;     // [USTAGES] unpack written + TMA landed
  uint64_t* u_empty = u_full + USTAGES;     // [USTAGES] MMA done reading
  uint64_t* acc_full = u_empty + USTAGES;   // [NBUF]
  uint64_t* acc_empty = acc_full + NBUF;    // [NBUF]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + NBUF);
  uint32_t* unpack_flag = tmem_slot + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = K / kBK;
  const int G = K / 64;
  const bool dump = !B_PACKED && partials != nullptr;
  const int has_lr = (!dump && rank_pad > 0) ? 1 : 0;
  // the low-rank operands take one ring slot per 64 ranks (128-byte rows)
  const int lr_slots = has_lr ? (rank_pad + 63) / 64 : 0;
  // Persistent: this CTA takes tiles blockIdx.x, +gridDim.x, ... (N-tile
  // fastest). Ring slots and TMEM group buffers are counted across tiles, so
  // the next tile's loads and MMAs start while this tile's epilogue finishes.
  const int tiles_n = N / BN;
  const int ntiles = ((M + kBM - 1) / kBM) * tiles_n;

  for (int i = threadIdx.x; i < ZERO_BYTES / 16; i += THREADS)
    reinterpret_cast<uint4*>(zero)[i] = make_uint4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int i = 0; i < PSTAGES; ++i) { mbar_init(&p_full[i], 1); mbar_init(&p_empty[i], 1); }
    for (int i = 0; i < USTAGES; ++i) {
      mbar_init(&u_full[i], UNPACK ? 2 : 1);
      mbar_init(&u_empty[i], 1);
    }
    for (int i = 0; i < NBUF; ++i) { mbar_init(&acc_full[i], 1); mbar_init(&acc_empty[i], EPI_WARPS); }
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

  // register hand-off. Packed activations: the launch gives 512 x 128 =
  // 65536 registers; warpgroups 0-1 (producer, MMA, unpack) drop to 56 (14336)
  // and the two epilogue warpgroups rise to 200 (51200). Otherwise 384 x 168 =
  // 64512; warpgroup 0 (producer, MMA, two unpack warps or idle) drops to 56
  // (7168) and the epilogue rises to 224 (57344).
  if (warp < EPI0) {
    regs_dec<56>();
    if (warp == 0 && lane == 0) {
      // -------------------------------------------------------------- TMA
      int ui = 0, pk = 0;   // operand-ring and packed-ring slots used so far
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      const int m0 = (tile / tiles_n) * kBM, n0 = (tile % tiles_n) * BN;
      for (int h = 0; h < lr_slots; ++h, ++ui) {
        // low-rank operands (ranks 64h .. 64h+63) go straight into an operand ring slot
        const int u = ui % USTAGES;
        ok = mbar_wait(&u_empty[u], ((ui / USTAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER);
        if (!ok) break;
        mbar_arrive_expect_tx(&u_full[u], kBM * 128 + BN * 128);
        if (UNPACK) mbar_arrive(&u_full[u]);
        uint8_t* us = ustage + u * USTAGE_BYTES;
        tma_load_2d(us, &tmLA, &u_full[u], 64 * h, m0);
        tma_load_2d(us + UA_BYTES, &tmUP, &u_full[u], 64 * h, n0);
      }
      if (!ok) break;
      for (int kb = 0; kb < nk; ++kb, ++ui) {
        if (UNPACK) {
          const int s = pk % PSTAGES;
          if (!mbar_wait(&p_empty[s], ((pk / PSTAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* ps = pstage + s * (PA + PB);
          mbar_arrive_expect_tx(&p_full[s], PA + PB);
          if (A_PACKED) tma_load_2d(ps, &tmA, &p_full[s], kb * (kBK / 2), m0);
          if (B_PACKED) tma_load_2d(ps + PA, &tmB, &p_full[s], kb * (kBK / 2), n0);
          ++pk;
        }
        GWB_TRACE_AT(0, ui);
        const int u = ui % USTAGES;
        if (!mbar_wait(&u_empty[u], ((ui / USTAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        uint8_t* us = ustage + u * USTAGE_BYTES;
        const uint32_t tx = (A_PACKED ? 0u : (uint32_t)UA_BYTES) +
                            (B_PACKED ? 0u : (uint32_t)UB_BYTES) + (dump ? 0u : SCALE_BYTES);
        mbar_arrive_expect_tx(&u_full[u], tx);
        if (!A_PACKED) tma_load_2d(us, &tmA, &u_full[u], kb * kBK, m0);
        if (!B_PACKED) tma_load_2d(us + UA_BYTES, &tmB, &u_full[u], kb * kBK, n0);
        if (!dump) {
          // scale area: [A g0 | A g1 | B]; B = the stored 8-group rows
          // (B_PACKED) or the two groups' one-hot rows
          uint8_t* so = us + UA_BYTES + UB_BYTES;
#pragma unroll
          for (int gs = 0; gs < 2; ++gs)
            tma_load_2d(so + gs * SOPA, &tmAS, &u_full[u], 0, (2 * kb + gs) * M + m0);
          if (B_PACKED) {
            tma_load_2d(so + 2 * SOPA, &tmBS, &u_full[u], 8 * (kb >> 2), n0);
          } else {
#pragma unroll
            for (int gs = 0; gs < 2; ++gs)
              tma_load_2d(so + 2 * SOPA + gs * SOPB, &tmBS, &u_full[u], 0, (2 * kb + gs) * N + n0);
          }
        }
      }
      }
    } else if (warp == 1 && lane == 0) {
      // -------------------------------------------------------------- MMA
      constexpr uint32_t idesc = idesc_fmt0_f32(kBM, BN);      // e4m3 x e4m3 -> f32
      constexpr uint32_t idesc_lr = idesc_bf16(kBM, BN);
      constexpr uint32_t idesc_s = idesc_fmt0_f32(kBM, BN);    // f16 x f16 -> f32
      const uint32_t zero_addr = smem_u32(zero);
      bool ok = true;
      int ui = 0, gi = 0;   // operand-ring slots and group buffers used so far
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
      if (has_lr) {
        // the tile's first group slot <- la · proj_upᵀ (f32), 64 ranks per ring slot
        const int b = gi % NBUF;
        for (int h = 0; h < lr_slots; ++h, ++ui) {
          const int u = ui % USTAGES;
          ok = mbar_wait(&u_full[u], (ui / USTAGES) & 1, GWB_ERR_TIMEOUT_MMA) &&
               (h > 0 || mbar_wait(&acc_empty[b], ((gi / NBUF) & 1) ^ 1, GWB_ERR_TIMEOUT_MMA));
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(ustage + u * USTAGE_BYTES), b_base = a_base + UA_BYTES;
          const int nk16 = min(4, (rank_pad - 64 * h) / 16);
          for (int k = 0; k < nk16; ++k)
            mma_f16(tmem + b * BN, sdesc_k128(a_base + 32 * k), sdesc_k128(b_base + 32 * k),
                    idesc_lr, (h > 0 || k > 0) ? 1u : 0u);
          mma_commit(&u_empty[u]);
        }
        if (!ok) break;
        mma_commit(&acc_full[b]);
        ++gi;
      }
      for (int kb = 0; kb < nk && ok; ++kb, ++ui) {
        const int u = ui % USTAGES;
        if (!mbar_wait(&u_full[u], (ui / USTAGES) & 1, GWB_ERR_TIMEOUT_MMA)) { ok = false; break; }
        GWB_TRACE_AT(1, ui);
        tc_fence_after();
        const uint32_t a_base = smem_u32(ustage + u * USTAGE_BYTES);
        const uint32_t b_base = a_base + UA_BYTES;
        const uint32_t s_base = b_base + UB_BYTES;
        for (int gs = 0; gs < 2 && ok; ++gs, ++gi) {
          const int b = gi % NBUF;
          if (!mbar_wait(&acc_empty[b], ((gi / NBUF) & 1) ^ 1, GWB_ERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          GWB_TRACE_AT(2, gi);
          tc_fence_after();
          const uint32_t d = tmem + b * BN;
          mma_f8(d, sdesc_k128(a_base + 64 * gs), sdesc_k128(b_base + 64 * gs), idesc, 0u);
          mma_f8(d, sdesc_k128(a_base + 64 * gs + 32), sdesc_k128(b_base + 64 * gs + 32), idesc,
                 1u);
          if (!dump) {
            // S_b = a_scale[:, g] ⊗ w_scale[:, g], exact in f32 (11-bit x 11-bit)
            const uint32_t sa = s_base + gs * SOPA;
            const uint32_t sb = s_base + 2 * SOPA + (B_PACKED ? 0 : gs * SOPB);
            mma_f16(tmem + NBUF * BN + b * BN, sdesc_scale(sa, zero_addr - sa),
                    sdesc_scale(sb, zero_addr - sb), idesc_s, 0u);
          }
          mma_commit(&acc_full[b]);
        }
        mma_commit(&u_empty[u]);
      }
      }
    } else if (UNPACK && warp >= 2) {
      // -------------------------------------------------------------- unpack
      const int tid = threadIdx.x - 64;
      int ui = 0, pk = 0;
      bool live = true;
      for (int tile = blockIdx.x; live && tile < ntiles; tile += gridDim.x) {
      ui += lr_slots;   // the low-rank slots are filled by the TMA thread alone
      for (int kb = 0; kb < nk; ++kb, ++ui, ++pk) {
        const int s = pk % PSTAGES;
        const int u = ui % USTAGES;
        // one thread waits, the named barrier broadcasts the outcome so all
        // unpack warps always leave the loop together
        if (tid == 0) {
          bool ok = mbar_wait(&p_full[s], (pk / PSTAGES) & 1, GWB_ERR_TIMEOUT_UNPACK);
          ok = ok && mbar_wait(&u_empty[u], ((ui / USTAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_UNPACK);
          *unpack_flag = ok ? 1u : 0u;
        }
        asm volatile("bar.sync 1, %0;" ::"n"(UNPACK_THREADS) : "memory");
        if (*reinterpret_cast<volatile uint32_t*>(unpack_flag) == 0u) { live = false; break; }
        if (tid == 0) GWB_TRACE_AT(3, ui);
        const uint8_t* ps = pstage + s * (PA + PB);
        uint8_t* us = ustage + u * USTAGE_BYTES;
        if (A_PACKED) unpack_tile<kBM, UNPACK_THREADS>(ps, us, tid);
        if (B_PACKED) unpack_tile<BN, UNPACK_THREADS>(ps + PA, us + UA_BYTES, tid);
        fence_proxy_async_smem();
        asm volatile("bar.sync 1, %0;" ::"n"(UNPACK_THREADS) : "memory");
        if (tid == 0) {
          GWB_TRACE_AT(4, ui);
          mbar_arrive(&p_empty[s]);
          mbar_arrive(&u_full[u]);
        }
      }
      }
    }
  } else {
    if constexpr (A_PACKED) regs_inc<200>();
    else regs_inc<224>();
    // ---------------------------------------------------------------- epilogue
    // Per group: load the f32 group sum V (= 2^-18 * v, exact) of this warp's
    // 32 rows x EC columns and the scale product S = a_scale * w_scale the
    // tensor core wrote beside it, wait once, hand the TMEM buffer straight
    // back to the MMA warp, then acc += V * S (one FFMA per element; acc is
    // 2^-18 times the result until the end of the tile). Epilogue warps
    // EPI0..EPI0+7: lane quarter warp % 4 (tile rows 32*(warp%4)..), column
    // slice ((warp-EPI0)/4)*EC.
    const int q = warp & 3;
    const int cb = ((warp - EPI0) >> 2) * EC;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
    const int total = G + has_lr;
    bool ok = true;
    int gi = 0;   // group buffers consumed so far (counted across tiles)
    for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
    const int m0 = (tile / tiles_n) * kBM, n0 = (tile % tiles_n) * BN;
    const int row = m0 + 32 * q + lane;
    const bool rv = row < M;
    float2 acc[EC / 2];
#pragma unroll
    for (int j = 0; j < EC / 2; ++j) acc[j] = make_float2(0.f, 0.f);
    for (int gt = 0; gt < total; ++gt, ++gi) {
      const int b = gi % NBUF;
      if (!mbar_wait(&acc_full[b], (gi / NBUF) & 1, GWB_ERR_TIMEOUT_EPILOGUE)) { ok = false; break; }
      if (warp == EPI0 && lane == 0) GWB_TRACE_AT(5, gi);
      tc_fence_after();
      const uint32_t col0 = lane_base + b * BN + cb;
      const bool lr = has_lr && gt == 0;
      uint32_t v[EC], sc[EC];
#pragma unroll
      for (int c = 0; c < EC; c += 32) tmem_ld32(col0 + c, v + c);
      if (!lr && !dump) {
#pragma unroll
        for (int c = 0; c < EC; c += 32) tmem_ld32(col0 + NBUF * BN + c, sc + c);
      }
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (warp == EPI0 && lane == 0) GWB_TRACE_AT(6, gi);
      if (lr) {
        // f32 low-rank product la·proj_upᵀ seeds the accumulator (in its scale)
#pragma unroll
        for (int j = 0; j < EC; j += 2)
          acc[j / 2] = make_float2(__uint_as_float(v[j]) * kRescale,
                                   __uint_as_float(v[j + 1]) * kRescale);
      } else if (dump) {
        if (rv) {
          const int g = gt - has_lr;
          uint4* dp = reinterpret_cast<uint4*>(partials + ((size_t)g * M + row) * N + n0 + cb);
#pragma unroll
          for (int j = 0; j < EC / 4; ++j)
            dp[j] = make_uint4(
                (uint32_t)__float2int_rn(__uint_as_float(v[4 * j]) * kUnscale),
                (uint32_t)__float2int_rn(__uint_as_float(v[4 * j + 1]) * kUnscale),
                (uint32_t)__float2int_rn(__uint_as_float(v[4 * j + 2]) * kUnscale),
                (uint32_t)__float2int_rn(__uint_as_float(v[4 * j + 3]) * kUnscale));
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
          f[j] = acc[(c + j) / 2].x * kUnscale;
          f[j + 1] = acc[(c + j) / 2].y * kUnscale;
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
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, TMEM_COLS);
}

// ======================================================================
// NVFP4 (the reference's SVDQuant format): kind::mxf4nvf4 block-scaled MMA
// ======================================================================
// Activations and weights are packed e2m1 codes with e4m3 scales per
// 16-element block in the cuBLAS blocked layout (exactly the reference's
// `weight` / `weight_scale` buffers and its quantiser output); the tensor
// core applies the block scales itself. Tile 128 x 256, persistent. Per
// k-block of 256 codes: TMA brings the 128 x 128-byte A and 256 x 128-byte B
// tiles (SWIZZLE_128B) and three 2 KB bulk copies bring the blocked scale
// tiles (A rows, B rows 0-127, B rows 128-255); the MMA thread copies each
// 128 x 4 scale tile into TMEM (tcgen05.cp) and issues four K = 64 MMAs.
// The low-rank product is issued first into the same accumulator, in the
// accumulator's units (divided by s2 * weight_scale_2[n]) and exact to
// ~2^-17: the quantiser writes la3 = [u_hi | u_lo | u_hi] with u = bf16(x ·
// proj_down) / s2 split into two bf16 parts, the load-time form of the
// up-projection is up3 = [w_hi | w_hi | w_lo] with w = proj_up[n] /
// weight_scale_2[n] split alike, and la3 · up3ᵀ = u_hi w_hi + u_lo w_hi +
// u_hi w_lo (the u_lo w_lo term is below 2^-17). Both are TMA-loaded. The
// epilogue is y = acc * s2 * weight_scale_2[n] + bias.
namespace nv4 {
constexpr int BN = 256;
constexpr int KB_BYTES = 128;                 // packed bytes of one k-block row (256 codes)
constexpr int STAGES = 4;
constexpr int A_BYTES = kBM * KB_BYTES;       // 16 KB
constexpr int B_BYTES = BN * KB_BYTES;        // 32 KB
constexpr int SFA_BYTES = 4 * 512;            // four 128 x 4 blocked scale tiles
constexpr int SFB_BYTES = 2 * SFA_BYTES;      // two 128-row groups
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;   // 54 KB
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
constexpr int TMEM_COLS = 512;
constexpr int ACC_COL = 0, SF_COL = 256;
constexpr int SF_SLOT = 48;                   // SFA 16 columns + SFB 32 columns
constexpr int SF_SLOTS = 4;
constexpr int THREADS = 384;                  // warp 0 TMA, 1 MMA, 4-11 epilogue
constexpr int EPI0 = 4;
constexpr int EPI_WARPS = 8;
constexpr int EC = BN / 2;
}  // namespace nv4

static_assert(nv4::SMEM_BYTES <= 232448, "NVFP4 shared memory exceeds 227 KB");
static_assert(nv4::SF_COL + nv4::SF_SLOTS * nv4::SF_SLOT <= nv4::TMEM_COLS, "TMEM overflow");

__global__ void __launch_bounds__(nv4::THREADS, 1)
gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmLA, const __grid_constant__ CUtensorMap tmUP,
                  const uint8_t* __restrict__ a_sblk, const uint8_t* __restrict__ w_sblk,
                  const float* __restrict__ a_work, const float* __restrict__ w_scale_2,
                  int ws2_per_channel, const __nv_bfloat16* __restrict__ bias,
                  __nv_bfloat16* __restrict__ out, int M, int N, int K, int rank_pad) {
  using namespace nv4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 1;
  uint64_t* sf_full = acc_empty + 1;          // [SF_SLOTS] scale tiles copied into TMEM
  uint64_t* sf_empty = sf_full + SF_SLOTS;    // [SF_SLOTS] MMAs reading the slot done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sf_empty + SF_SLOTS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = K / 256;
  const int ncb = K / 64;                     // blocked-layout tile columns per 128 rows
  const int has_lr = rank_pad > 0 ? 1 : 0;
  // the three-part low-rank operands (K = 3 * rank_pad) take one ring stage
  // per 64 of K (128-byte rows)
  const int lr_k = 3 * rank_pad;
  const int lr_slots = has_lr ? (lr_k + 63) / 64 : 0;
  // N % 256 == 128: the last N tile is half a tile (B rows past N read as
  // zeros by TMA; their scale tiles are not loaded and their columns not stored)
  const int tiles_n = (N + BN - 1) / BN;
  const int ntiles = ((M + kBM - 1) / kBM) * tiles_n;

  if (threadIdx.x == 0) {
    // a stage is free again once the MMA thread and the scale-copy thread
    // have both released it
    for (int i = 0; i < STAGES; ++i) { mbar_init(&full[i], 1); mbar_init(&empty[i], 2); }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, EPI_WARPS);
    for (int i = 0; i < SF_SLOTS; ++i) { mbar_init(&sf_full[i], 1); mbar_init(&sf_empty[i], 1); }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) { tmem_alloc(tmem_slot, TMEM_COLS); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < EPI0) {
    regs_dec<48>();
    if (warp == 0 && lane < 4) {
      // -------------------------------------------------------------- TMA
      // lane 0 A (and the low-rank operands), lane 1 B, lane 2 A scales,
      // lane 3 the two groups of B scales
      const int pl = lane;
      int ui = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        const int mt = tile / tiles_n, m0 = mt * kBM, n0 = (tile % tiles_n) * BN;
        const bool half_n = n0 + 128 >= N;   // only B rows n0 .. n0+127 exist
        for (int h = 0; h < lr_slots; ++h, ++ui) {
          const int u = ui % STAGES;
          ok = mbar_wait(&empty[u], ((ui / STAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER);
          ok = __all_sync(0xFu, ok);
          if (!ok) break;
          if (pl == 0) {
            // columns 64h .. 64h+63 of la3 and up3
            uint8_t* us = smem + u * STAGE_BYTES;
            mbar_arrive_expect_tx(&full[u], kBM * 128 + BN * 128);
            tma_load_2d(us, &tmLA, &full[u], 64 * h, m0);
            tma_load_2d(us + A_BYTES, &tmUP, &full[u], 64 * h, n0);
          }
          __syncwarp(0xFu);
        }
        if (!ok) break;
        for (int kb = 0; kb < nk; ++kb, ++ui) {
          const int u = ui % STAGES;
          ok = mbar_wait(&empty[u], ((ui / STAGES) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER);
          if (!__all_sync(0xFu, ok)) break;
          if (pl == 0)
            mbar_arrive_expect_tx(&full[u], half_n ? STAGE_BYTES - SFA_BYTES : STAGE_BYTES);
          __syncwarp(0xFu);
          uint8_t* us = smem + u * STAGE_BYTES;
          uint8_t* sfa = us + A_BYTES + B_BYTES;
          if (pl == 0) {
            tma_load_2d(us, &tmA, &full[u], kb * KB_BYTES, m0);
          } else if (pl == 1) {
            tma_load_2d(us + A_BYTES, &tmB, &full[u], kb * KB_BYTES, n0);
          } else if (pl == 2) {
            bulk_load(sfa, a_sblk + ((size_t)mt * ncb + 4 * kb) * 512, SFA_BYTES, &full[u]);
          } else {
            const size_t rb = (size_t)(n0 / 128);
            bulk_load(sfa + SFA_BYTES, w_sblk + (rb * ncb + 4 * kb) * 512, SFA_BYTES, &full[u]);
            if (!half_n)
              bulk_load(sfa + 2 * SFA_BYTES, w_sblk + ((rb + 1) * ncb + 4 * kb) * 512, SFA_BYTES,
                        &full[u]);
          }
        }
      }
    } else if (warp == 1 && lane == 0) {
      // -------------------------------------------------------------- MMA
      constexpr uint32_t idesc = idesc_mxf4(kBM, BN);
      constexpr uint32_t idesc_lr = idesc_bf16(kBM, BN);
      int ui = 0, lt = 0, kbi = 0;   // ring stages, tiles, k-blocks (scale slots) used
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x, ++lt) {
        if (!mbar_wait(acc_empty, (lt & 1) ^ 1, GWB_ERR_TIMEOUT_MMA)) break;
        tc_fence_after();
        for (int h = 0; h < lr_slots; ++h, ++ui) {
          // acc <- la3 · up3ᵀ, one ring stage per 64 of K
          const int u = ui % STAGES;
          ok = mbar_wait(&full[u], (ui / STAGES) & 1, GWB_ERR_TIMEOUT_MMA);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + u * STAGE_BYTES), b_base = a_base + A_BYTES;
          const int nk16 = min(4, (lr_k - 64 * h) / 16);
          for (int k = 0; k < nk16; ++k)
            mma_f16(tmem + ACC_COL, sdesc_k128(a_base + 32 * k), sdesc_k128(b_base + 32 * k),
                    idesc_lr, (h > 0 || k > 0) ? 1u : 0u);
          mma_commit(&empty[u]);
        }
        if (!ok) break;
        for (int kb = 0; kb < nk; ++kb, ++ui, ++kbi) {
          const int u = ui % STAGES;
          const int sl = kbi % SF_SLOTS;
          if (!mbar_wait(&full[u], (ui / STAGES) & 1, GWB_ERR_TIMEOUT_MMA) ||
              !mbar_wait(&sf_full[sl], (kbi / SF_SLOTS) & 1, GWB_ERR_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + u * STAGE_BYTES);
          const uint32_t b_base = a_base + A_BYTES;
          const uint32_t sfa_t = tmem + SF_COL + sl * SF_SLOT, sfb_t = sfa_t + 16;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma_mxf4(tmem + ACC_COL, sdesc_k128(a_base + 32 * ks), sdesc_k128(b_base + 32 * ks),
                     idesc, sfa_t + 4 * ks, sfb_t + 8 * ks,
                     (has_lr || kb > 0 || ks > 0) ? 1u : 0u);
          mma_commit(&empty[u]);
          mma_commit(&sf_empty[sl]);
        }
        if (ok) mma_commit(acc_full);
      }
    } else if (warp == 2 && lane == 0) {
      // ----------------------------------------------------- scale copies
      // Copies each k-block's blocked scale tiles from its ring stage into a
      // TMEM scale slot (tcgen05.cp), up to SF_SLOTS k-blocks ahead of the
      // MMA thread, so the copies stay out of the MMA issue stream. The MMA
      // thread waits sf_full (this thread's commit: copies done) before the
      // stage's MMAs and releases the slot with its own commit (sf_empty).
      // This thread follows every use of every ring stage, the low-rank ones
      // included, and releases each (empty counts both threads): a parity
      // wait cannot tell a stage's completions apart when the waiter runs a
      // phase ahead or two behind.
      int ui = 0, kbi = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < ntiles; tile += gridDim.x) {
        for (int h = 0; h < lr_slots; ++h, ++ui) {
          const int u = ui % STAGES;
          ok = mbar_wait(&full[u], (ui / STAGES) & 1, GWB_ERR_TIMEOUT_PRODUCER);
          if (!ok) break;
          mbar_arrive(&empty[u]);
        }
        if (!ok) break;
        for (int kb = 0; kb < nk; ++kb, ++ui, ++kbi) {
          const int u = ui % STAGES;
          const int sl = kbi % SF_SLOTS;
          if (!mbar_wait(&full[u], (ui / STAGES) & 1, GWB_ERR_TIMEOUT_PRODUCER) ||
              !mbar_wait(&sf_empty[sl], ((kbi / SF_SLOTS) & 1) ^ 1, GWB_ERR_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sfa_s = smem_u32(smem + u * STAGE_BYTES) + A_BYTES + B_BYTES;
          const uint32_t sfb_s = sfa_s + SFA_BYTES;
          const uint32_t sfa_t = tmem + SF_COL + sl * SF_SLOT, sfb_t = sfa_t + 16;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            // per K = 64 step: A scales 4 columns, B scales 8 columns (rows
            // n / 32: the first 128-row group in 0-3, the second in 4-7)
            tmem_cp_32x128b_x4(sfa_t + 4 * ks, sdesc_noswz(sfa_s + 512 * ks, 0));
            tmem_cp_32x128b_x4(sfb_t + 8 * ks, sdesc_noswz(sfb_s + 512 * ks, 0));
            tmem_cp_32x128b_x4(sfb_t + 8 * ks + 4, sdesc_noswz(sfb_s + SFA_BYTES + 512 * ks, 0));
          }
          mma_commit(&sf_full[sl]);
          mma_commit(&empty[u]);
        }
      }
    }
  } else {
    regs_inc<224>();
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const int cb = ((warp - EPI0) >> 2) * EC;
    const float s2 = a_work[1];
    int lt = 0;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++lt) {
      const int m0 = (tile / tiles_n) * kBM, n0 = (tile % tiles_n) * BN;
      if (!mbar_wait(acc_full, lt & 1, GWB_ERR_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      uint32_t v[EC];
      const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) + ACC_COL + cb;
#pragma unroll
      for (int c = 0; c < EC; c += 32) tmem_ld32(base + c, v + c);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
      const int row = m0 + 32 * q + lane;
      if (row >= M || n0 + cb >= N) continue;
      uint4* op = reinterpret_cast<uint4*>(out + (size_t)row * N + n0 + cb);
#pragma unroll
      for (int c = 0; c < EC; c += 8) {
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float w2 = ws2_per_channel ? __ldg(w_scale_2 + n0 + cb + c + j) : __ldg(w_scale_2);
          f[j] = __uint_as_float(v[c + j]) * (s2 * w2);
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
        op[c / 8] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
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

// Streaming multiprocessors of the current device (persistent grids).
static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  return n;
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_gemm_w8a8(const W8A8Args& a, bool fp8, cudaStream_t st) {
  if (a.M <= 0 || a.K <= 0 || a.K % kBK || a.N % w8::BN) return GWB_E_SHAPE;
  if (!a.a_q || !a.a_scale || !a.w_q || !a.w_scale || !a.out) return GWB_E_SHAPE;
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
    cudaFuncSetAttribute(gemm_w8a8_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         w8::SMEM_BYTES);
    cudaFuncSetAttribute(gemm_w8a8_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         w8::SMEM_BYTES);
    attr = true;
  }
  const int n_sm = sm_count();
  const int ntiles = ((a.M + kBM - 1) / kBM) * (a.N / w8::BN);
  const int grid = ntiles < n_sm ? ntiles : n_sm;
  auto kern = fp8 ? gemm_w8a8_kernel<true> : gemm_w8a8_kernel<false>;
  kern<<<grid, w8::THREADS, w8::SMEM_BYTES, st>>>(
      tA, tB, a.a_scale, a.w_scale, static_cast<const __nv_bfloat16*>(a.bias),
      static_cast<__nv_bfloat16*>(a.out), a.M, a.N, a.K, a.gelu);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

template <bool A_PACKED, bool B_PACKED, int BN>
static int launch_gemm_w4a4_cfg(const W4A4Args& a, cudaStream_t st) {
  using C = w4::Cfg<A_PACKED, B_PACKED, BN>;
  const int G = a.K / 64;
  CUtensorMap tA, tB, tAS, tBS, tLA, tUP;
  int rc = A_PACKED ? make_tmap(&tA, a.a_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K / 2, a.M,
                               kBK / 2, kBM, CU_TENSOR_MAP_SWIZZLE_NONE)
                     : make_tmap(&tA, a.a_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K, a.M, kBK,
                                 kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = B_PACKED ? make_tmap(&tB, a.w_q8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K / 2, a.N, kBK / 2,
                            BN, CU_TENSOR_MAP_SWIZZLE_NONE)
                : make_tmap(&tB, a.w_q8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K, a.N, kBK, BN,
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
    // stored weight scales f16 [N, G] (8 groups per box row), or the
    // one-hot rows f16 [G, N, 8]
    rc = B_PACKED ? make_tmap(&tBS, a.w_scale_k8, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, G, a.N, 8,
                              BN, CU_TENSOR_MAP_SWIZZLE_NONE)
                  : make_tmap(&tBS, a.w_scale_k8, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, 8,
                              (uint64_t)G * a.N, 8, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  if (a.rank_pad > 0 && !a.partials) {
    rc = make_tmap(&tLA, a.la, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.rank_pad, a.M, 64, kBM,
                   CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap(&tUP, a.up, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.rank_pad, a.N, 64, BN,
                   CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  auto kern = gemm_w4a4_kernel<A_PACKED, B_PACKED, BN>;
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    attr = true;
  }
  const int ntiles = ((a.M + kBM - 1) / kBM) * (a.N / BN);
  const int n_sm = sm_count();
  const int grid = ntiles < n_sm ? ntiles : n_sm;
  kern<<<grid, w4::threads<A_PACKED>(), C::SMEM_BYTES, st>>>(
      tA, tB, tAS, tBS, tLA, tUP, static_cast<const __nv_bfloat16*>(a.bias),
      static_cast<__nv_bfloat16*>(a.out), a.partials, a.M, a.N, a.K,
      a.partials ? 0 : a.rank_pad, a.gelu);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

int launch_gemm_w4a4(const W4A4Args& a, bool a_packed, bool b_packed, cudaStream_t st) {
  if (a.M <= 0 || a.K <= 0 || a.K % kBK || a.N % 128) return GWB_E_SHAPE;
  if (a.rank_pad < 0 || a.rank_pad > 128 || a.rank_pad % 16) return GWB_E_SHAPE;
  if (a.rank_pad > 0 && !a.partials && (!a.la || !a.up)) return GWB_E_SHAPE;
  if (!a.partials && !a.out) return GWB_E_SHAPE;
  if (!a.a_codes || !a.w_q8) return GWB_E_SHAPE;
  if (!a.partials && (!a.a_scale_k8 || !a.w_scale_k8)) return GWB_E_SHAPE;
  if (b_packed && a.partials) return GWB_E_SHAPE;
  const int G = a.K / 64;
  if ((int64_t)G * a.M > 0x7fffffff || (int64_t)G * a.N > 0x7fffffff) return GWB_E_SHAPE;
  if (!al16(a.a_codes) || !al16(a.w_q8) || (a.out && !al16(a.out)) ||
      (a.bias && !al16(a.bias)) ||
      (a.la && !al16(a.la)) || (a.up && !al16(a.up)) || (a.partials && !al16(a.partials)) ||
      (!a.partials && (!al16(a.a_scale_k8) || !al16(a.w_scale_k8))))
    return GWB_E_ALIGN;
  // stored weight scales [N, G]: each row must start on a 16-byte boundary
  if (b_packed && (G % 8)) return GWB_E_SHAPE;
  // tile 128 x 128: a 64-wide tile (four TMEM group buffers) measured half
  // the throughput, the per-group issue and hand-off latency being fixed
  if (a_packed && b_packed) return launch_gemm_w4a4_cfg<true, true, 128>(a, st);
  if (a_packed) return launch_gemm_w4a4_cfg<true, false, 128>(a, st);
  if (b_packed) return launch_gemm_w4a4_cfg<false, true, 128>(a, st);
  return launch_gemm_w4a4_cfg<false, false, 128>(a, st);
}

int launch_gemm_nvfp4(const NvFp4Args& a, cudaStream_t st) {
  if (a.M <= 0 || a.K <= 0 || a.K % 256 || a.N <= 0 || a.N % 128) return GWB_E_SHAPE;
  if (a.rank_pad < 0 || a.rank_pad > 128 || a.rank_pad % 16) return GWB_E_SHAPE;
  if (a.rank_pad > 0 && (!a.la || !a.up)) return GWB_E_SHAPE;
  if (!a.a_codes || !a.w_codes || !a.a_sblk || !a.w_sblk || !a.a_work || !a.w_scale_2 || !a.out)
    return GWB_E_SHAPE;
  if (!al16(a.a_codes) || !al16(a.w_codes) || !al16(a.a_sblk) || !al16(a.w_sblk) ||
      !al16(a.out) || (a.bias && !al16(a.bias)) || (a.la && !al16(a.la)) ||
      (a.up && !al16(a.up)) || (reinterpret_cast<uintptr_t>(a.a_work) & 7u) ||
      (reinterpret_cast<uintptr_t>(a.w_scale_2) & 3u))
    return GWB_E_ALIGN;
  CUtensorMap tA, tB, tLA, tUP;
  int rc = make_tmap(&tA, a.a_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K / 2, a.M,
                     nv4::KB_BYTES, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = make_tmap(&tB, a.w_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.K / 2, a.N, nv4::KB_BYTES,
                 nv4::BN, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  tLA = tA;
  tUP = tB;
  if (a.rank_pad > 0) {
    rc = make_tmap(&tLA, a.la, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3 * a.rank_pad, a.M, 64, kBM,
                   CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = make_tmap(&tUP, a.up, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 3 * a.rank_pad, a.N, 64,
                   nv4::BN, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  static bool attr = false;
  if (!attr) {
    cudaFuncSetAttribute(gemm_nvfp4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         nv4::SMEM_BYTES);
    attr = true;
  }
  const int ntiles = ((a.M + kBM - 1) / kBM) * ((a.N + nv4::BN - 1) / nv4::BN);
  const int n_sm = sm_count();
  gemm_nvfp4_kernel<<<ntiles < n_sm ? ntiles : n_sm, nv4::THREADS, nv4::SMEM_BYTES, st>>>(
      tA, tB, tLA, tUP, static_cast<const uint8_t*>(a.a_sblk),
      static_cast<const uint8_t*>(a.w_sblk), a.a_work, a.w_scale_2, a.ws2_per_channel,
      static_cast<const __nv_bfloat16*>(a.bias), static_cast<__nv_bfloat16*>(a.out), a.M, a.N,
      a.K, a.rank_pad);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

int launch_w4a4_weight_expand(const void* w_codes, void* w_q8, int64_t N, int64_t K,
                              cudaStream_t st) {
  if (N <= 0 || K <= 0 || K % 64) return GWB_E_SHAPE;
  if ((reinterpret_cast<uintptr_t>(w_codes) & 3u) || (reinterpret_cast<uintptr_t>(w_q8) & 7u))
    return GWB_E_ALIGN;
  const int64_t nwords = N * K / 8;
  int64_t blocks = (nwords + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  w4a4_weight_expand_kernel<<<(int)blocks, 256, 0, st>>>(
      static_cast<const uint32_t*>(w_codes), static_cast<uint2*>(w_q8), nwords);
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
