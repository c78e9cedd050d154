// C-ABI entry points of libgwb200.so (declared in include/gwb200.h). The
// library is one translation unit: the kernel sources are included here.
#include <cuda_runtime.h>
#include <cstdio>
#include <cstring>
#include "gwb.h"
#include "ptx.cuh"
#include "act_quant.cu"
#include "gemm.cu"
#include "codec.cu"
#include "awq.cu"
#include "../../include/gwb200.h"

#ifndef GWB_ARCH_STRING
#define GWB_ARCH_STRING "sm_100a"
#endif

namespace {

__global__ void probe_add_one_kernel(const float* __restrict__ x, float* __restrict__ y,
                                     int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = x[i] + 1.0f;
}

inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

// A wait that can never complete, run with the kernels' own bounded wait:
// every warp waits on an mbarrier nothing arrives on while the CTA holds
// TMEM, exactly as a GEMM role waits on its pipeline. Each wait gives up
// after gwb_wait_limit cycles and records `code` in gwb_dev_error; the CTA
// then meets at a barrier and frees its TMEM, so the context stays usable.
__global__ void stalled_wait_kernel(int code) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    gwb::mbar_init(&bar, 1);
    gwb::fence_barrier_init();
  }
  if (warp == 0) {
    gwb::tmem_alloc(&slot, 32);
    gwb::tmem_relinquish();
  }
  gwb::tc_fence_before();
  __syncthreads();
  gwb::tc_fence_after();
  if (lane == 0) (void)gwb::mbar_wait(&bar, 0, code);
  gwb::tc_fence_before();
  __syncthreads();
  if (warp == 0) gwb::tmem_dealloc(slot, 32);
}

inline bool fits_int(int64_t v) { return v >= 0 && v <= 0x7fffffff; }

inline int check_w4a4_shape(int64_t M, int64_t N, int64_t K, int rank_pad) {
  if (!fits_int(M) || !fits_int(N) || !fits_int(K) || M == 0) return GWB_E_SHAPE;
  if (K % 128 || N % 128) return GWB_E_SHAPE;
  if (rank_pad < 0 || rank_pad > 128 || rank_pad % 16) return GWB_E_SHAPE;
  return GWB_SUCCESS;
}

inline bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int gwb_build_info(char* buf, size_t len) {
  int rt = 0;
  cudaRuntimeGetVersion(&rt);
  char tmp[160];
  int n = snprintf(tmp, sizeof(tmp), "gwb200 cuda_runtime=%d.%d archs=%s", rt / 1000,
                   (rt % 1000) / 10, GWB_ARCH_STRING);
  if (buf && len) {
    strncpy(buf, tmp, len - 1);
    buf[len - 1] = '\0';
  }
  return n;
}

int gwb_probe_add_one(const float* x, float* y, int64_t n, void* stream) {
  if (n < 0) return GWB_E_SHAPE;
  if (n == 0) return GWB_SUCCESS;
  int blocks = (int)((n + 255) / 256);
  if (blocks > 4096) blocks = 4096;
  probe_add_one_kernel<<<blocks, 256, 0, S(stream)>>>(x, y, n);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

int gwb_svdq_w4a4_quant(const void* x, const void* smooth, const void* proj_down_t, int64_t M,
                        int64_t K, int rank_pad, void* codes, void* ascale, void* la,
                        void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(M) || !fits_int(K) || K % 64) return GWB_E_SHAPE;
  if (rank_pad < 0 || rank_pad > 128 || rank_pad % 16) return GWB_E_SHAPE;
  if (rank_pad > 0 && (!proj_down_t || !la)) return GWB_E_SHAPE;
  if (!x || !codes || !ascale) return GWB_E_SHAPE;
  if (!al16(x) || !al16(codes) || (smooth && !al16(smooth)) ||
      (proj_down_t && !al16(proj_down_t)) || (la && !al16(la)) ||
      (reinterpret_cast<uintptr_t>(ascale) & 1u))
    return GWB_E_ALIGN;
  return gwb::launch_act_int4(x, smooth, rank_pad ? proj_down_t : nullptr, codes, ascale,
                              rank_pad ? la : nullptr, (int)M, (int)K, rank_pad, false, S(stream));
}

int gwb_svdq_w4a4_quant_mma(const void* x, const void* smooth, const void* proj_down_t,
                            int64_t M, int64_t K, int rank_pad, void* a_q8, void* a_scale_k8,
                            void* la, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(M) || !fits_int(K) || K % 64 || (K / 64) * M > 0x7fffffff) return GWB_E_SHAPE;
  if (rank_pad < 0 || rank_pad > 128 || rank_pad % 16) return GWB_E_SHAPE;
  if (rank_pad > 0 && (!proj_down_t || !la)) return GWB_E_SHAPE;
  if (!x || !a_q8 || !a_scale_k8) return GWB_E_SHAPE;
  if (!al16(x) || !al16(a_q8) || !al16(a_scale_k8) || (smooth && !al16(smooth)) ||
      (proj_down_t && !al16(proj_down_t)) || (la && !al16(la)))
    return GWB_E_ALIGN;
  return gwb::launch_act_int4(x, smooth, rank_pad ? proj_down_t : nullptr, a_q8, a_scale_k8,
                              rank_pad ? la : nullptr, (int)M, (int)K, rank_pad, true, S(stream));
}

int gwb_svdq_w4a4_scale_k8(const void* scale, int64_t R, int64_t K, void* scale_k8,
                           void* stream) {
  if (R == 0) return GWB_SUCCESS;
  if (!fits_int(R) || !fits_int(K) || K % 64 || (K / 64) * R > 0x7fffffff) return GWB_E_SHAPE;
  if (!scale || !scale_k8) return GWB_E_SHAPE;
  if ((reinterpret_cast<uintptr_t>(scale) & 1u) || !al16(scale_k8)) return GWB_E_ALIGN;
  return gwb::launch_scale_k8(scale, scale_k8, (int)R, (int)K, S(stream));
}

int gwb_svdq_w4a4_weight_expand(const void* w_codes, int64_t N, int64_t K, void* w_q8,
                                void* stream) {
  if (N == 0) return GWB_SUCCESS;
  if (!fits_int(N) || !fits_int(K)) return GWB_E_SHAPE;
  if (!w_codes || !w_q8) return GWB_E_SHAPE;
  return gwb::launch_w4a4_weight_expand(w_codes, w_q8, N, K, S(stream));
}

int gwb_svdq_w4a4_gemm(const void* a_q8, const void* a_scale_k8, const void* w_q8,
                       const void* w_scale_k8, const void* la, const void* proj_up,
                       const void* bias, int64_t M, int64_t N, int64_t K, int rank_pad, int gelu,
                       void* out, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  int rc = check_w4a4_shape(M, N, K, rank_pad);
  if (rc) return rc;
  gwb::W4A4Args a{a_q8, a_scale_k8, w_q8, w_scale_k8, la, proj_up, bias, out, nullptr,
                  (int)M, (int)N, (int)K, rank_pad, gelu ? 1 : 0};
  return gwb::launch_gemm_w4a4(a, false, false, S(stream));
}

int gwb_svdq_w4a4_gemm_packed(const void* codes, const void* a_scale_k8, const void* w_q8,
                              const void* w_scale_k8, const void* la, const void* proj_up,
                              const void* bias, int64_t M, int64_t N, int64_t K, int rank_pad,
                              int gelu, void* out, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  int rc = check_w4a4_shape(M, N, K, rank_pad);
  if (rc) return rc;
  gwb::W4A4Args a{codes, a_scale_k8, w_q8, w_scale_k8, la, proj_up, bias, out, nullptr,
                  (int)M, (int)N, (int)K, rank_pad, gelu ? 1 : 0};
  return gwb::launch_gemm_w4a4(a, true, false, S(stream));
}

int gwb_svdq_w4a4_group_partials(const void* codes, const void* w_q8, int64_t M, int64_t N,
                                 int64_t K, int32_t* partials, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  int rc = check_w4a4_shape(M, N, K, 0);
  if (rc) return rc;
  if ((K / 64) * M * N > (int64_t)1 << 31) return GWB_E_CAPACITY;
  gwb::W4A4Args a{codes, nullptr, w_q8, nullptr, nullptr, nullptr, nullptr, nullptr,
                  partials, (int)M, (int)N, (int)K, 0, 0};
  return gwb::launch_gemm_w4a4(a, true, false, S(stream));
}

int gwb_svdq_w4a4_linear(const void* x, const void* smooth, const void* proj_down_t,
                         const void* w_q8, const void* w_scale_k8, const void* proj_up,
                         const void* bias, int64_t M, int64_t N, int64_t K, int rank_pad,
                         int gelu, void* a_q8, void* a_scale_k8, void* la, void* out,
                         void* stream) {
  if (M == 0) return GWB_SUCCESS;
  int rc = check_w4a4_shape(M, N, K, rank_pad);
  if (rc) return rc;
  rc = gwb_svdq_w4a4_quant_mma(x, smooth, proj_down_t, M, K, rank_pad, a_q8, a_scale_k8, la,
                               stream);
  if (rc) return rc;
  return gwb_svdq_w4a4_gemm(a_q8, a_scale_k8, w_q8, w_scale_k8, la, proj_up, bias, M, N, K,
                            rank_pad, gelu, out, stream);
}

int gwb_svdq_w4a4_gemm_stored(const void* a_q8, const void* a_scale_k8, const void* w_codes,
                              const void* w_scale, const void* la, const void* proj_up,
                              const void* bias, int64_t M, int64_t N, int64_t K, int rank_pad,
                              int gelu, void* out, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  int rc = check_w4a4_shape(M, N, K, rank_pad);
  if (rc) return rc;
  gwb::W4A4Args a{a_q8, a_scale_k8, w_codes, w_scale, la, proj_up, bias, out, nullptr,
                  (int)M, (int)N, (int)K, rank_pad, gelu ? 1 : 0};
  return gwb::launch_gemm_w4a4(a, false, true, S(stream));
}

int gwb_svdq_w4a4_gemm_packed_stored(const void* codes, const void* a_scale_k8,
                                     const void* w_codes, const void* w_scale, const void* la,
                                     const void* proj_up, const void* bias, int64_t M, int64_t N,
                                     int64_t K, int rank_pad, int gelu, void* out, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  int rc = check_w4a4_shape(M, N, K, rank_pad);
  if (rc) return rc;
  gwb::W4A4Args a{codes, a_scale_k8, w_codes, w_scale, la, proj_up, bias, out, nullptr,
                  (int)M, (int)N, (int)K, rank_pad, gelu ? 1 : 0};
  return gwb::launch_gemm_w4a4(a, true, true, S(stream));
}

int gwb_svdq_w4a4_linear_stored(const void* x, const void* smooth, const void* proj_down_t,
                                const void* w_codes, const void* w_scale, const void* proj_up,
                                const void* bias, int64_t M, int64_t N, int64_t K, int rank_pad,
                                int gelu, void* a_q8, void* a_scale_k8, void* la, void* out,
                                void* stream) {
  if (M == 0) return GWB_SUCCESS;
  int rc = check_w4a4_shape(M, N, K, rank_pad);
  if (rc) return rc;
  rc = gwb_svdq_w4a4_quant_mma(x, smooth, proj_down_t, M, K, rank_pad, a_q8, a_scale_k8, la,
                               stream);
  if (rc) return rc;
  return gwb_svdq_w4a4_gemm_stored(a_q8, a_scale_k8, w_codes, w_scale, la, proj_up, bias, M, N, K,
                                   rank_pad, gelu, out, stream);
}

int gwb_w8a8_quant(const void* x, int64_t M, int64_t K, void* q, void* scale, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(M) || !fits_int(K) || K % 8 || K == 0) return GWB_E_SHAPE;
  if (!x || !q || !scale) return GWB_E_SHAPE;
  if (!al16(x) || !al16(q) || (reinterpret_cast<uintptr_t>(scale) & 3u)) return GWB_E_ALIGN;
  return gwb::launch_act_int8(x, q, scale, (int)M, (int)K, S(stream));
}

int gwb_w8a8_gemm(const void* q, const float* scale, const void* w_q, const float* w_scale,
                  const void* bias, int64_t M, int64_t N, int64_t K, int gelu, void* out,
                  void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(M) || !fits_int(N) || !fits_int(K)) return GWB_E_SHAPE;
  gwb::W8A8Args a{q, scale, w_q, w_scale, bias, out, (int)M, (int)N, (int)K, gelu ? 1 : 0};
  return gwb::launch_gemm_w8a8(a, false, S(stream));
}

int gwb_w8a8_linear(const void* x, const void* w_q, const float* w_scale, const void* bias,
                    int64_t M, int64_t N, int64_t K, int gelu, void* q, void* scale, void* out,
                    void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(N) || K % 128 || N % 256) return GWB_E_SHAPE;
  int rc = gwb_w8a8_quant(x, M, K, q, scale, stream);
  if (rc) return rc;
  return gwb_w8a8_gemm(q, static_cast<const float*>(scale), w_q, w_scale, bias, M, N, K, gelu,
                       out, stream);
}

int gwb_fp8_quant(const void* x, int64_t M, int64_t K, void* q, void* scale, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(M) || !fits_int(K) || K % 8 || K == 0) return GWB_E_SHAPE;
  if (!x || !q || !scale) return GWB_E_SHAPE;
  if (!al16(x) || !al16(q) || (reinterpret_cast<uintptr_t>(scale) & 3u)) return GWB_E_ALIGN;
  return gwb::launch_act_fp8(x, q, scale, (int)M, (int)K, S(stream));
}

int gwb_fp8_gemm(const void* q, const float* scale, const void* w_q, const float* w_scale,
                 const void* bias, int64_t M, int64_t N, int64_t K, int gelu, void* out,
                 void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(M) || !fits_int(N) || !fits_int(K)) return GWB_E_SHAPE;
  gwb::W8A8Args a{q, scale, w_q, w_scale, bias, out, (int)M, (int)N, (int)K, gelu ? 1 : 0};
  return gwb::launch_gemm_w8a8(a, true, S(stream));
}

int gwb_fp8_linear(const void* x, const void* w_q, const float* w_scale, const void* bias,
                   int64_t M, int64_t N, int64_t K, int gelu, void* q, void* scale, void* out,
                   void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(N) || K % 128 || N % 256) return GWB_E_SHAPE;
  int rc = gwb_fp8_quant(x, M, K, q, scale, stream);
  if (rc) return rc;
  return gwb_fp8_gemm(q, static_cast<const float*>(scale), w_q, w_scale, bias, M, N, K, gelu,
                      out, stream);
}

int gwb_nvfp4_quant(const void* x, const void* smooth, int64_t M, int64_t K, void* codes,
                    void* sblk, float* work, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(M) || !fits_int(K) || K % 64 || K == 0) return GWB_E_SHAPE;
  if (!x || !codes) return GWB_E_SHAPE;
  if (!al16(x) || !al16(codes) || (smooth && !al16(smooth)) || !sblk || !work || !al16(work))
    return GWB_E_ALIGN;
  return gwb::launch_act_nvfp4(x, smooth, work, codes, sblk, (int)M, (int)K, S(stream));
}

int gwb_nvfp4_quant_lowrank(const void* x, const void* smooth, const void* down_t, int64_t M,
                            int64_t K, int rank_pad, void* codes, void* sblk, float* work,
                            void* la, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(M) || !fits_int(K) || K % 64 || K == 0) return GWB_E_SHAPE;
  if (rank_pad < 16 || rank_pad > 128 || rank_pad % 16) return GWB_E_SHAPE;
  if (!x || !codes || !down_t) return GWB_E_SHAPE;
  if (!al16(x) || !al16(codes) || (smooth && !al16(smooth)) || !sblk || !work || !al16(work) ||
      !al16(down_t) || !la)
    return GWB_E_ALIGN;
  return gwb::launch_act_nvfp4_lowrank(x, smooth, down_t, work, codes, sblk, la, (int)M, (int)K,
                                       rank_pad, S(stream));
}

int gwb_nvfp4_gemm(const void* a_codes, const void* a_sblk, const float* a_work,
                   const void* w_codes, const void* w_sblk, const float* w_scale_2,
                   int ws2_per_channel, const void* la, const void* proj_up, const void* bias,
                   int64_t M, int64_t N, int64_t K, int rank_pad, void* out, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(M) || !fits_int(N) || !fits_int(K)) return GWB_E_SHAPE;
  gwb::NvFp4Args a{a_codes, a_sblk, a_work, w_codes, w_sblk, w_scale_2, ws2_per_channel ? 1 : 0,
                   la, proj_up, bias, out, (int)M, (int)N, (int)K, rank_pad};
  return gwb::launch_gemm_nvfp4(a, S(stream));
}

int gwb_device_error(int* code) {
  if (!code) return GWB_E_SHAPE;
  if (cudaDeviceSynchronize() != cudaSuccess) return GWB_E_LAUNCH;
  return gwb::device_error_read_and_clear(code);
}

int gwb_nunchaku_qweight_to_e2m1(const void* qweight, int64_t N, int64_t K, void* weight) {
  if (N <= 0 || K <= 0 || N % 128 || K % 128) return GWB_E_SHAPE;
  if (((uintptr_t)qweight | (uintptr_t)weight) & 3u) return GWB_E_ALIGN;
  gwb::codec::qweight_to_e2m1(static_cast<const uint32_t*>(qweight), N, K,
                              static_cast<uint32_t*>(weight));
  return GWB_SUCCESS;
}

int gwb_nunchaku_wscales_to_blocked(const void* wscales, int64_t N, int64_t K, void* blocked) {
  if (N <= 0 || K <= 0 || N % 128 || K % 64) return GWB_E_SHAPE;
  gwb::codec::wscales_to_blocked(static_cast<const uint8_t*>(wscales), N, K,
                                 static_cast<uint8_t*>(blocked));
  return GWB_SUCCESS;
}

int gwb_nunchaku_vector_unpack(const void* vec, int64_t n, int elem_bytes, void* out) {
  if (n <= 0 || n % 128) return GWB_E_SHAPE;
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
    return GWB_E_SHAPE;
  gwb::codec::vector_unpack(static_cast<const uint8_t*>(vec), n, elem_bytes,
                            static_cast<uint8_t*>(out));
  return GWB_SUCCESS;
}

int gwb_nunchaku_lowrank_unpack(const void* w, int64_t rows, int64_t rank, int down, void* out) {
  if (rows <= 0 || rank <= 0 || rows % 16 || rank % 16) return GWB_E_SHAPE;
  gwb::codec::lowrank_unpack(static_cast<const uint16_t*>(w), rows, rank, down != 0,
                             static_cast<uint16_t*>(out));
  return GWB_SUCCESS;
}

int gwb_lowrank_dequant(const void* q, const float* scale, int64_t rows, int64_t cols,
                        int block_dim, int scheme, void* out) {
  if (rows <= 0 || cols <= 0 || (block_dim != 0 && block_dim != 1)) return GWB_E_SHAPE;
  if ((block_dim == 0 ? rows : cols) % 32) return GWB_E_SHAPE;
  if (scheme != 0 && scheme != 1) return GWB_E_SHAPE;
  gwb::codec::lowrank_dequant(static_cast<const uint8_t*>(q), scale, rows, cols, block_dim,
                              scheme == 1, static_cast<uint16_t*>(out));
  return GWB_SUCCESS;
}

int gwb_awq_qweight_unpack(const void* qweight, int64_t N, int64_t K, void* weight) {
  if (N <= 0 || K <= 0 || N % 4 || K % 64) return GWB_E_SHAPE;
  gwb::codec::awq_qweight_unpack(static_cast<const uint16_t*>(qweight), N, K,
                                 static_cast<uint8_t*>(weight));
  return GWB_SUCCESS;
}

int gwb_awq_w4a16_mm(const void* x, const void* weight, const void* wscales, const void* wzeros,
                     const void* bias, int64_t M, int64_t N, int64_t K, void* out,
                     void* stream) {
  if (M == 0) return GWB_SUCCESS;
  if (!fits_int(M) || !fits_int(N) || !fits_int(K) || N % 16 || K % 128 || N == 0)
    return GWB_E_SHAPE;
  if (!x || !weight || !wscales || !wzeros || !out) return GWB_E_SHAPE;
  if (!al16(x) || !al16(weight)) return GWB_E_ALIGN;
  const cudaError_t e = gwb::launch_awq_w4a16(
      static_cast<const __nv_bfloat16*>(x), static_cast<const uint8_t*>(weight),
      static_cast<const __nv_bfloat16*>(wscales), static_cast<const __nv_bfloat16*>(wzeros),
      static_cast<const __nv_bfloat16*>(bias), static_cast<__nv_bfloat16*>(out), (int)M, (int)N,
      (int)K, S(stream));
  return e == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

int gwb_set_wait_limit(long long cycles) {
  const long long v = cycles > 0 ? cycles : (long long)GWB_WAIT_LIMIT_CYCLES;
  return cudaMemcpyToSymbol(gwb_wait_limit, &v, sizeof(v)) == cudaSuccess ? GWB_SUCCESS
                                                                          : GWB_E_LAUNCH;
}

int gwb_test_stalled_wait(int code, void* stream) {
  if (code <= 0) return GWB_E_SHAPE;
  stalled_wait_kernel<<<2, 128, 0, S(stream)>>>(code);
  return cudaGetLastError() == cudaSuccess ? GWB_SUCCESS : GWB_E_LAUNCH;
}

int gwb_device_check(void) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GWB_E_ARCH;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return (major == 10 && minor == 0) ? GWB_SUCCESS : GWB_E_ARCH;
}

const char* gwb_status_string(int status) {
  switch (status) {
    case GWB_SUCCESS: return "success";
    case GWB_E_SHAPE: return "unsupported or inconsistent sizes";
    case GWB_E_ALIGN: return "pointer not 16-byte aligned";
    case GWB_E_LAUNCH: return "kernel launch failed";
    case GWB_E_TMAP: return "TMA tensor-map encode failed";
    case GWB_E_DRIVER: return "driver entry point cuTensorMapEncodeTiled unavailable";
    case GWB_E_DEVICE: return "device-side bounded wait expired";
    case GWB_E_ARCH: return "device is not sm_100 (B200)";
    case GWB_E_CAPACITY: return "request exceeds a fixed capacity";
    default: return "unknown status";
  }
}

}  // extern "C"

// The no-allocation variant of gwb_svdq_w4a4_linear (its own file: the scratch
// array and the host code that looks up its address live together).
#include "noalloc.cu"
