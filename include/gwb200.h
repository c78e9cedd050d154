/* gwb200 — C ABI of the B200 (sm_100a) SVDQuant quantized-linear hot path.
 *
 * Plain pointers and sizes only; every compute entry point enqueues work on
 * the given CUDA stream (cudaStream_t passed as void*; NULL = legacy default
 * stream), never synchronises, never allocates, and returns a GwbStatus code
 * (0 = success). Device buffers must be 16-byte aligned and row-major
 * contiguous. G = K/64 groups.
 *
 * INT4 codes (activations and weights alike):
 *   codes        u8   [R, K/2]   sign-magnitude nibbles (bit 3 = sign,
 *                                bits 0-2 = |q|, q in -7..7), even k low
 * Group scales, interchange form (checkpoints, module buffers, quant output):
 *   scale        f16  [R, G]     one scale per 64-group
 * INT4 codes, GEMM operand form (weights: gwb_svdq_w4a4_weight_expand at
 * load time; activations: gwb_svdq_w4a4_quant_mma):
 *   q8 (w_q8, a_q8) u8 [R, K]    each code as the e4m3 byte of q * 2^-9,
 *                                elements of every 8-block in the order
 *                                0 2 4 6 1 3 5 7
 * Group scales, GEMM scale-operand rows (gwb_svdq_w4a4_scale_k8 converts,
 * gwb_svdq_w4a4_quant_mma writes them directly):
 *   scale_k8     f16  [G, R, 8]  group g's scale at k = g mod 8, zeros at
 *                                the other seven k
 * Other tensors:
 *   x            bf16 [M, K];  smooth bf16 [K] (or NULL)
 *   proj_down_t  bf16 [rank_pad, K]   (L1 transposed; rows >= rank are zero)
 *   la           bf16 [M, rank_pad]   x·L1 on raw x
 *   proj_up      bf16 [N, rank_pad];  bias bf16 [N] (or NULL);  out bf16 [M, N]
 * Constraints: K % 128 == 0; N % 128 == 0 (W4A4) / N % 256 == 0 (W8A8);
 * rank_pad a multiple of 16, at most 128.
 */
#ifndef GWB200_H
#define GWB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces `build_info` (reference csrc/cozy_kernels/ops.cpp:24-27): torch
 * pin replaced by the CUDA runtime version and fatbin arch. Writes a NUL-
 * terminated string; returns its length. */
int gwb_build_info(char* buf, size_t len);

/* Replaces `probe_add_one` (reference csrc/cozy_kernels/probe.cu:9-27;
 * registered at csrc/cozy_kernels/ops.cpp:29-36): y = x + 1 on `n` floats. */
int gwb_probe_add_one(const float* x, float* y, int64_t n, void* stream);

/* Replaces `cozy_gen_worker::svdq_quant(x2, smooth, s2, blocked)`
 * (reference src/gen_worker/models/svdq_fused.py:293-296, kernel :116-155)
 * fused with the low-rank down-projection `la = x2 @ proj_down`
 * (svdq_fused.py:524, svdq_native.py:153). INT4 group-64 with fp16 scales in
 * place of NVFP4; no per-tensor second-level scale. Writes the packed
 * interchange form (codes [M, K/2], ascale [M, G]). */
int gwb_svdq_w4a4_quant(const void* x, const void* smooth, const void* proj_down_t,
                        int64_t M, int64_t K, int rank_pad,
                        void* codes, void* ascale, void* la, void* stream);

/* The same quantiser (identical codes and scales) writing the GEMM operand
 * form: a_q8 [M, K] and a_scale_k8 [G, M, 8]. The hot-path producer of
 * `SvdqLinear.forward` (svdq_native.py:145-147). */
int gwb_svdq_w4a4_quant_mma(const void* x, const void* smooth, const void* proj_down_t,
                            int64_t M, int64_t K, int rank_pad,
                            void* a_q8, void* a_scale_k8, void* la, void* stream);

/* Group scales f16 [R, G] -> scale-operand rows f16 [G, R, 8] (weights at
 * load time, or activation scales from gwb_svdq_w4a4_quant). Counterpart of
 * the reference's load-time scale repack `to_blocked_scales`
 * (nvfp4_quant.py:72-84). */
int gwb_svdq_w4a4_scale_k8(const void* scale, int64_t R, int64_t K, void* scale_k8,
                           void* stream);

/* Load-time weight repack (counterpart of the reference's load-time
 * `to_buffers` / `pack_e2m1` repacks, svdq_layout.py:473-483): packed INT4
 * w_codes u8 [N, K/2] -> w_q8 u8 [N, K] in the GEMM operand form. */
int gwb_svdq_w4a4_weight_expand(const void* w_codes, int64_t N, int64_t K, void* w_q8,
                                void* stream);

/* Replaces `cozy_gen_worker::svdq_gemm_w4a4_lora(qa, sa, wq_kn, ws, s2,
 * second, lora_act, up, bias)` (reference svdq_fused.py:379-383, kernel
 * :180-238) and the baseline chain `_gemm_w4a4` + scale + low-rank + bias of
 * `SvdqLinear.forward` (svdq_native.py:148-155). Both operands in GEMM
 * operand form, both scales as scale-operand rows; gelu != 0 applies
 * GELU(tanh) after the bias. */
int gwb_svdq_w4a4_gemm(const void* a_q8, const void* a_scale_k8, const void* w_q8,
                       const void* w_scale_k8, const void* la, const void* proj_up,
                       const void* bias, int64_t M, int64_t N, int64_t K, int rank_pad,
                       int gelu, void* out, void* stream);

/* The same GEMM taking the activations as packed INT4 codes [M, K/2] (the
 * interchange form, e.g. from gwb_svdq_w4a4_quant): TMA loads the packed
 * tiles and the kernel unpacks them to the operand layout in shared memory
 * (the reference's `svdq_gemm_w4a4_lora` takes packed `qa`, svdq_fused.py:
 * 379-383). */
int gwb_svdq_w4a4_gemm_packed(const void* codes, const void* a_scale_k8, const void* w_q8,
                              const void* w_scale_k8, const void* la, const void* proj_up,
                              const void* bias, int64_t M, int64_t N, int64_t K, int rank_pad,
                              int gelu, void* out, void* stream);

/* Debug/parity entry (no reference counterpart beyond the group sums the
 * reference's GEMM forms internally, svdq_fused.py:213-222): the same
 * tcgen05 GEMM with the epilogue replaced by a dump of every 64-group integer
 * partial sum, partials s32 [G, M, N]. */
int gwb_svdq_w4a4_group_partials(const void* codes, const void* w_q8, int64_t M, int64_t N,
                                 int64_t K, int32_t* partials, void* stream);

/* Whole SvdqLinear forward (reference svdq_native.py:140-156): quantise to
 * operand form + GEMM. The caller supplies the scratch buffers a_q8 [M, K],
 * a_scale_k8 [G, M, 8] and la [M, rank_pad]. */
int gwb_svdq_w4a4_linear(const void* x, const void* smooth, const void* proj_down_t,
                         const void* w_q8, const void* w_scale_k8, const void* proj_up,
                         const void* bias, int64_t M, int64_t N, int64_t K, int rank_pad,
                         int gelu, void* a_q8, void* a_scale_k8, void* la, void* out,
                         void* stream);

/* Replaces `cozy_gen_worker::svdq_gemm_w4a4_lora(qa, sa, wq_kn, ws, ...)`
 * (reference svdq_fused.py:379-383) with the weight as stored: w_codes
 * u8 [N, K/2] packed INT4 and w_scale f16 [N, G] (the module's `weight` /
 * `weight_scale` buffers, no load-time repack). The kernel TMA-loads the
 * packed weight tiles and expands them to the e4m3 operand layout in shared
 * memory; the stored scale rows (8 groups per 16 bytes) are the B side of
 * the scale MMA, selected per group by the one-hot activation scale rows.
 * Activations in operand form (gwb_svdq_w4a4_quant_mma). G % 8 == 0
 * (K % 512 == 0). */
int gwb_svdq_w4a4_gemm_stored(const void* a_q8, const void* a_scale_k8, const void* w_codes,
                              const void* w_scale, const void* la, const void* proj_up,
                              const void* bias, int64_t M, int64_t N, int64_t K, int rank_pad,
                              int gelu, void* out, void* stream);

/* The same with the activations as packed codes [M, K/2] too (both operands
 * expanded in shared memory; a_scale_k8 from gwb_svdq_w4a4_scale_k8). */
int gwb_svdq_w4a4_gemm_packed_stored(const void* codes, const void* a_scale_k8,
                                     const void* w_codes, const void* w_scale, const void* la,
                                     const void* proj_up, const void* bias, int64_t M, int64_t N,
                                     int64_t K, int rank_pad, int gelu, void* out, void* stream);

/* Whole SvdqLinear forward (reference svdq_native.py:140-156) on the
 * weights as stored: gwb_svdq_w4a4_quant_mma into the caller's scratch
 * (a_q8 [M, K], a_scale_k8 [G, M, 8], la [M, rank_pad]), then
 * gwb_svdq_w4a4_gemm_stored. */
int gwb_svdq_w4a4_linear_stored(const void* x, const void* smooth, const void* proj_down_t,
                                const void* w_codes, const void* w_scale, const void* proj_up,
                                const void* bias, int64_t M, int64_t N, int64_t K, int rank_pad,
                                int gelu, void* a_q8, void* a_scale_k8, void* la, void* out,
                                void* stream);

/* No counterpart in the reference. The same computation as
 * gwb_svdq_w4a4_linear for callers that cannot allocate device memory (their
 * device memory belongs to another framework's pool or a fixed start-up
 * budget, or their serving loop forbids cudaMalloc once running): the
 * intermediates live in a 32 MiB array inside the library, held on every GPU
 * that loads it until exit. Needs M*K + M*(K/64)*16 + M*rank_pad*2 bytes
 * (each part rounded up to 256); larger calls return GWB_E_CAPACITY. Calls
 * share the array: work from calls that overlap on the GPU races. The first
 * call on a device looks up the array's address; make it before any stream
 * capture. The address is cached per process and device and is not looked
 * up again after a device reset. `stream` must belong to the current device
 * (another device's stream returns GWB_E_SHAPE). Allocates nothing. */
int gwb_svdq_w4a4_linear_noalloc(const void* x, const void* smooth, const void* proj_down_t,
                                 const void* w_q8, const void* w_scale_k8,
                                 const void* proj_up, const void* bias, int64_t M, int64_t N,
                                 int64_t K, int rank_pad, int gelu, void* out, void* stream);

/* Failure handling (counterpart of the reference's collective timeout and
 * stall detection, src/gen_worker/parallel/group.py:26, :265-285). Every
 * pipeline wait in the kernels is bounded: after `cycles` SM clock cycles it
 * records a GWB_ERR_TIMEOUT_* code (read with gwb_device_error), every role
 * unwinds, TMEM is freed and the kernel returns. cycles <= 0 restores the
 * default (4e9, ~2 s). */
int gwb_set_wait_limit(long long cycles);

/* Test entry (no reference counterpart): a kernel whose wait can never
 * complete (an mbarrier nothing arrives on, while it holds TMEM), so that
 * a test can make the bounded wait run out and check the recorded `code`
 * and that the next launch works. */
int gwb_test_stalled_wait(int code, void* stream);

/* Replaces the W8A8 activation quantiser `_quant_src` rowwise branch
 * (reference src/gen_worker/models/w8a8.py:261-273): per-token symmetric
 * INT8, q s8 [M, K], scale f32 [M]. */
int gwb_w8a8_quant(const void* x, int64_t M, int64_t K, void* q, void* scale, void* stream);

/* Replaces `torch._scaled_mm(xq, w.t(), scale_a, scale_b, bias)` rowwise in
 * `Fp8ScaledLinear.forward` (reference w8a8.py:374-378) with INT8 operands;
 * w_q s8 [N, K], w_scale f32 [N]; gelu != 0 fuses GELU(tanh). */
int gwb_w8a8_gemm(const void* q, const float* scale, const void* w_q, const float* w_scale,
                  const void* bias, int64_t M, int64_t N, int64_t K, int gelu, void* out,
                  void* stream);

/* Whole `Fp8ScaledLinear.forward` rowwise (reference w8a8.py:359-381) with
 * INT8: quantise into the caller's scratch q / scale, then GEMM. */
int gwb_w8a8_linear(const void* x, const void* w_q, const float* w_scale, const void* bias,
                    int64_t M, int64_t N, int64_t K, int gelu, void* q, void* scale,
                    void* out, void* stream);

/* The reference's own W8A8 number format, FP8 e4m3 rowwise. Replaces the
 * dynamic rowwise branch of `_quant_src` (reference w8a8.py:261-273):
 * scale f32 [M] = max(amax_row / 448, 1e-12); q = e4m3 bytes [M, K] of
 * clamp(bf16(x * bf16(1 / scale)), +-448), nearest-even. */
int gwb_fp8_quant(const void* x, int64_t M, int64_t K, void* q, void* scale, void* stream);

/* Replaces `torch._scaled_mm(xq, w.t(), scale_a, scale_b, bias)` rowwise in
 * `Fp8ScaledLinear.forward` (reference w8a8.py:374-378): w_q e4m3 bytes
 * [N, K] and w_scale f32 [N] as the reference's producer writes them
 * (`quantize_tree_w8a8`, w8a8.py:774-779); f32 accumulation; gelu != 0
 * fuses GELU(tanh). */
int gwb_fp8_gemm(const void* q, const float* scale, const void* w_q, const float* w_scale,
                 const void* bias, int64_t M, int64_t N, int64_t K, int gelu, void* out,
                 void* stream);

/* Whole `Fp8ScaledLinear.forward` rowwise (reference w8a8.py:359-381):
 * quantise into the caller's scratch q [M, K] / scale [M], then GEMM. */
int gwb_fp8_linear(const void* x, const void* w_q, const float* w_scale, const void* bias,
                   int64_t M, int64_t N, int64_t K, int gelu, void* q, void* scale,
                   void* out, void* stream);

/* The reference's own SVDQuant format, NVFP4 (e2m1 codes, e4m3 scales per
 * 16-element block in the cuBLAS blocked layout, fp32 second-level scale).
 * Replaces `quantize_activation` / `quantize_activation_torch` (reference
 * src/gen_worker/models/nvfp4_quant.py:92-103, 272-280) preceded by the
 * smoothing divide and the per-tensor `s2` of `SvdqLinear.forward`
 * (svdq_native.py:144-146): codes u8 [M, K/2] (element 2j in the low
 * nibble), sblk = blocked e4m3 scales (ceil(M/128)*128 * K/16 bytes, the
 * padding rows zero as in the reference), work f32 [4 + K] scratch (16-byte aligned;
 * work[1] = s2 on return). Bit-identical to the reference. K % 64 == 0. */
int gwb_nvfp4_quant(const void* x, const void* smooth, int64_t M, int64_t K, void* codes,
                    void* sblk, float* work, void* stream);

/* gwb_nvfp4_quant plus the low-rank down-projection of the same
 * `SvdqLinear.forward` (la = x2 @ proj_down on raw x, svdq_native.py:153),
 * computed in the pass that takes amax, so x is read twice instead of three
 * times: down_t bf16 [rank_pad, K] (proj_down transposed, zero-padded rows),
 * la: the three-part form bf16 [M, 3 * rank_pad] = [u_hi | u_lo | u_hi]
 * with u = bf16(x · proj_down) / s2 (f32 accumulation, then the bf16
 * rounding of the reference's matmul) split into two bf16 parts.
 * rank_pad a multiple of 16, at most 128; other arguments as
 * gwb_nvfp4_quant. */
int gwb_nvfp4_quant_lowrank(const void* x, const void* smooth, const void* down_t, int64_t M,
                            int64_t K, int rank_pad, void* codes, void* sblk, float* work,
                            void* la, void* stream);

/* Replaces `_gemm_w4a4` (`torch._scaled_mm` on float4_e2m1fn_x2 with blocked
 * scales, reference w4a4.py:173-180) and the rest of the NVFP4
 * `SvdqLinear.forward` (svdq_native.py:148-155): y = (A·B^T with block scales)
 * * s2 * w_scale_2[n] + la·proj_up^T + bias -> bf16 [M, N]. w_codes / w_sblk
 * / w_scale_2 are the reference module's `weight` / `weight_scale` /
 * `weight_scale_2` buffers as stored (w_scale_2 per channel [N] when
 * ws2_per_channel, else [1]). The low-rank branch shares the accumulator
 * in its units (divided by s2 * w_scale_2[n]): la = the three-part la3
 * [M, 3 * rank_pad] of gwb_nvfp4_quant_lowrank, proj_up = the three-part
 * up3 bf16 [N, 3 * rank_pad] = [w_hi | w_hi | w_lo], w = proj_up /
 * w_scale_2[n] split into two bf16 parts (load time); la3 · up3ᵀ keeps the
 * product to ~2^-17. K % 256 == 0, N % 128 == 0, rank_pad <= 128. */
int gwb_nvfp4_gemm(const void* a_codes, const void* a_sblk, const float* a_work,
                   const void* w_codes, const void* w_sblk, const float* w_scale_2,
                   int ws2_per_channel, const void* la, const void* proj_up, const void* bias,
                   int64_t M, int64_t N, int64_t K, int rank_pad, void* out, void* stream);

/* ---- Load-time codec: nunchaku "v1 single-file" SVDQuant tensors -> the
 * NVFP4 lane's buffers as stored. Host-memory functions (no GPU needed).
 * Together they replace `decode_linear` + `to_buffers` (reference
 * src/gen_worker/models/svdq_layout.py:363-438, 473-483) without the
 * logical-domain intermediate; GWB_E_SHAPE for sizes the format forbids. */

/* qweight I8 [N, K/2] (fragment interleave, svdq_layout.py:89-110) ->
 * `weight` u8 [N, K/2], packed e2m1 with element 2j in the low nibble
 * (pack_e2m1, nvfp4_quant.py:54-56). N % 128 == 0, K % 128 == 0; both
 * buffers 4-byte aligned. */
int gwb_nunchaku_qweight_to_e2m1(const void* qweight, int64_t N, int64_t K, void* weight);

/* wscales E4M3 [K/16, N] (micro-scale pack, svdq_layout.py:117-129) ->
 * `weight_scale` in the cuBLAS blocked layout (to_blocked_scales,
 * nvfp4_quant.py:72-84), N * K/16 bytes. N % 128 == 0, K % 64 == 0. */
int gwb_nunchaku_wscales_to_blocked(const void* wscales, int64_t N, int64_t K, void* blocked);

/* pack_scale vector (wcscales, smooth_factor, bias; svdq_layout.py:132-142)
 * of n elements of elem_bytes (1, 2, 4 or 8) -> row-major. n % 128 == 0. */
int gwb_nunchaku_vector_unpack(const void* vec, int64_t n, int elem_bytes, void* out);

/* pack_lowrank_weight-packed 16-bit factor (svdq_layout.py:145-162):
 * down = 1: proj_down [rows = in_features, rank] -> row-major [in, rank];
 * down = 0: proj_up [rows = out_features, rank] -> row-major [out, rank].
 * rows % 16 == 0, rank % 16 == 0. */
int gwb_nunchaku_lowrank_unpack(const void* w, int64_t rows, int64_t rank, int down, void* out);

/* Quantized low-rank factor (dequantize_lowrank, svdq_layout.py:284-306):
 * q [rows, cols] int8 (scheme 0) or e4m3 (scheme 1), fp32 scales per
 * 32-element block along block_dim (0: [rows/32, cols], 1: [rows, cols/32])
 * -> bf16 [rows, cols] = bf16(q * scale), round to nearest even. */
int gwb_lowrank_dequant(const void* q, const float* scale, int64_t rows, int64_t cols,
                        int block_dim, int scheme, void* out);

/* ---- AWQ W4A16 modulation layers (timestep-embedding consumers). */

/* qweight I32 [N/4, K/2] (TinyChat pack, reference svdq_awq.py:31-47) ->
 * `weight` u8 [N, K/2], unsigned 4-bit codes, element 2j in the low nibble
 * (the packed-resident module's buffer, svdq_awq_packed.py:262). Host
 * memory. N % 4 == 0, K % 64 == 0. */
int gwb_awq_qweight_unpack(const void* qweight, int64_t N, int64_t K, void* weight);

/* Replaces `cozy_gen_worker::awq_w4a16_mm` (svdq_awq_packed.py:51-103):
 * out bf16 [M, N] = x bf16 [M, K] · bf16(q * wscales + wzeros)^T + bias,
 * q the codes of `weight` u8 [N, K/2], wscales / wzeros bf16 [N, K/64]
 * (group 64, zeros pre-scaled and pre-negated), bias bf16 [N] or NULL; f32
 * accumulation. The dequantised weight is q * s + z rounded once to bf16,
 * equal to the reference's decode (`dequantize_w4x16` in f32, then bf16)
 * whenever q * s + z fits 24 significant bits. N % 16 == 0, K % 128 == 0,
 * x and weight 16-byte aligned. M == 0 is a no-op. */
int gwb_awq_w4a16_mm(const void* x, const void* weight, const void* wscales, const void* wzeros,
                     const void* bias, int64_t M, int64_t N, int64_t K, void* out, void* stream);

/* Reads and clears the device-side error flag set by a bounded wait that
 * expired (0 = none; 1 TMA producer, 2 MMA thread, 3 epilogue, 4 unpack
 * warps, 5 the INT4 quantiser's x boxes). Synchronises the device. */
int gwb_device_error(int* code);

/* 0 when the current device is sm_100 (B200), GWB_E_ARCH otherwise. */
int gwb_device_check(void);

/* Static description of a status code. */
const char* gwb_status_string(int status);

#ifdef __cplusplus
}
#endif

#endif /* GWB200_H */
