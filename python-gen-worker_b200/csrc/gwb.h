// Internal declarations shared by the CUDA translation units.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

// Host-visible status codes (also returned through the C ABI).
enum GwbStatus : int {
  GWB_SUCCESS = 0,
  GWB_E_SHAPE = 1,      // unsupported / inconsistent sizes
  GWB_E_ALIGN = 2,      // pointer not 16-byte aligned
  GWB_E_LAUNCH = 3,     // kernel launch failed
  GWB_E_TMAP = 4,       // tensor-map encode failed
  GWB_E_DRIVER = 5,     // driver entry point unavailable
  GWB_E_DEVICE = 6,     // device-side error flag was set (bounded wait expired)
  GWB_E_ARCH = 7,       // device is not sm_100
  GWB_E_CAPACITY = 8,   // request exceeds a fixed capacity
};

namespace gwb {
int launch_act_int4(const void* x, const void* smooth, const void* down_t, void* codes,
                    void* ascale, void* la, int M, int K, int rank_pad, bool mma_form,
                    cudaStream_t st);
int launch_scale_k8(const void* scale, void* scale_k8, int R, int K, cudaStream_t st);
int launch_act_int8(const void* x, void* q, void* scale, int M, int K, cudaStream_t st);
int launch_act_fp8(const void* x, void* q, void* scale, int M, int K, cudaStream_t st);
// NVFP4 activations: work f32 [4 + K], 16-byte aligned (work[0] amax scratch,
// work[1] = s2 out, work[4..] the smoothing reciprocals); codes u8 [M, K/2]; sblk = blocked
// e4m3 scales (padding rows written as zeros).
int launch_act_nvfp4(const void* x, const void* smooth, float* work, void* codes, void* sblk,
                     int M, int K, cudaStream_t st);
// la: the three-part la3 bf16 [M, 3 * rank_pad] (see act_nvfp4_kernel)
int launch_act_nvfp4_lowrank(const void* x, const void* smooth, const void* down_t, float* work,
                             void* codes, void* sblk, void* la, int M, int K, int rank_pad,
                             cudaStream_t st);

struct NvFp4Args {
  const void* a_codes;     // u8 [M, K/2] packed e2m1 (element 2j low nibble)
  const void* a_sblk;      // e4m3 block scales, cuBLAS blocked layout
  const float* a_work;     // f32 [2]; [1] = activation second-level scale s2
  const void* w_codes;     // u8 [N, K/2]
  const void* w_sblk;      // e4m3 block scales, blocked layout
  const float* w_scale_2;  // f32 [1] or [N]
  int ws2_per_channel;
  const void* la;          // bf16 [M, 3 * rank_pad] three-part la3 (quantiser), or null
  const void* up;          // bf16 [N, 3 * rank_pad] three-part up3 (load time), or null
  const void* bias;        // bf16 [N] or null
  void* out;               // bf16 [M, N]
  int M, N, K, rank_pad;
};
int launch_gemm_nvfp4(const NvFp4Args& a, cudaStream_t st);

struct W4A4Args {
  const void* a_codes;     // u8 [M, K/2] packed INT4 (a_packed) or u8 [M, K] operand form
  const void* a_scale_k8;  // f16 [K/64, M, 8] (group g's scale at k = g mod 8)
  const void* w_q8;        // u8 [N, K] expanded weight (launch_w4a4_weight_expand), or
                           // the stored packed weight u8 [N, K/2] (b_packed)
  const void* w_scale_k8;  // f16 [K/64, N, 8] one-hot rows, or the stored f16 [N, K/64] (b_packed)
  const void* la;          // bf16 [M, rank_pad] or null
  const void* up;          // bf16 [N, rank_pad] or null
  const void* bias;        // bf16 [N] or null
  void* out;               // bf16 [M, N]
  int32_t* partials;       // optional debug: s32 [K/64, M, N]; disables the epilogue
  int M, N, K, rank_pad, gelu;
};
int launch_gemm_w4a4(const W4A4Args& a, bool a_packed, bool b_packed, cudaStream_t st);
int launch_w4a4_weight_expand(const void* w_codes, void* w_q8, int64_t N, int64_t K,
                              cudaStream_t st);


struct W8A8Args {
  const void* a_q;        // s8 [M, K] (INT8) or e4m3 bytes [M, K] (FP8)
  const float* a_scale;   // f32 [M]
  const void* w_q;        // s8 [N, K]
  const float* w_scale;   // f32 [N]
  const void* bias;       // bf16 [N] or null
  void* out;              // bf16 [M, N]
  int M, N, K, gelu;
};
int launch_gemm_w8a8(const W8A8Args& a, bool fp8, cudaStream_t st);

int device_error_read_and_clear(int* code);
}  // namespace gwb
