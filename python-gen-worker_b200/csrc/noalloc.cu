// gwb_svdq_w4a4_linear_noalloc: the whole W4A4 linear for callers that cannot
// allocate device memory themselves.
//
// gwb_svdq_w4a4_linear needs three intermediate buffers between its two
// kernels (the INT4 codes and group scales in GEMM operand form, and the
// low-rank activation la) and expects
// the caller to allocate them. Some callers cannot: a host runtime whose
// device memory is owned by another framework's pool or by a fixed budget
// set at start-up, or a serving loop that forbids cudaMalloc/cudaFree (and
// the device-wide synchronisation they can cause) once it is running. This
// entry point keeps those intermediates in a fixed array that is part of the
// library image instead, so the caller passes only inputs and outputs.
//
// Limits and sharing:
//  * the array holds GWB_NOALLOC_SCRATCH_BYTES (32 MiB); every GPU on which
//    the library's device code is loaded keeps it until the process exits;
//  * a call needs M*K + M*(K/64)*16 + M*rank_pad*2 bytes (each part
//    rounded up to 256); larger calls return GWB_E_CAPACITY and do nothing;
//  * all calls on a device share the one array, and it keeps whatever the
//    last call wrote. Both kernels overwrite every scratch byte they later
//    read, so nothing has to be cleared between calls. Calls whose work
//    overlaps on the GPU (different streams without ordering, or several host
//    threads) race on the array and corrupt each other's results;
//  * the first call on each device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture begins. The address is cached per process and
//    per device, and is not looked up again after a device reset;
//  * `stream` must belong to the current device (the array's address is the
//    current device's); a stream of another device returns GWB_E_SHAPE.
#include <cuda_runtime.h>
#include <mutex>

#define GWB_NOALLOC_SCRATCH_BYTES (32ull << 20)
#define GWB_NOALLOC_MAX_DEVICES 64

// Host code must not use this name as a pointer: on the host it denotes a
// shadow symbol, not device memory. Its device address comes from
// cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char gwb_noalloc_scratch[GWB_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[GWB_NOALLOC_MAX_DEVICES] = {};

// Device address of the scratch array on the current device (looked up once
// per device, with that device current).
int noalloc_scratch(unsigned char** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return GWB_E_LAUNCH;
  if (dev < 0 || dev >= GWB_NOALLOC_MAX_DEVICES) return GWB_E_CAPACITY;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, gwb_noalloc_scratch) != cudaSuccess || p == nullptr)
      return GWB_E_LAUNCH;
    g_noalloc_ptr[dev] = p;
  }
  *out = static_cast<unsigned char*>(g_noalloc_ptr[dev]);
  return GWB_SUCCESS;
}

inline uint64_t round256(uint64_t v) { return (v + 255u) & ~uint64_t(255u); }

}  // namespace

extern "C" int gwb_svdq_w4a4_linear_noalloc(const void* x, const void* smooth,
                                            const void* proj_down_t, const void* w_q8,
                                            const void* w_scale_k8, const void* proj_up,
                                            const void* bias, int64_t M, int64_t N, int64_t K,
                                            int rank_pad, int gelu, void* out, void* stream) {
  if (M == 0) return GWB_SUCCESS;
  int rc = check_w4a4_shape(M, N, K, rank_pad);
  if (rc) return rc;
  const uint64_t codes_b = round256((uint64_t)M * (uint64_t)K);
  const uint64_t scale_b = round256((uint64_t)M * (uint64_t)(K / 64) * 16u);
  const uint64_t la_b = round256((uint64_t)M * (uint64_t)rank_pad * 2u);
  if (codes_b + scale_b + la_b > GWB_NOALLOC_SCRATCH_BYTES) return GWB_E_CAPACITY;
  if (!x || !w_q8 || !w_scale_k8 || !out) return GWB_E_SHAPE;
  if (stream != nullptr) {
    int cur = 0, sdev = 0;
    if (cudaGetDevice(&cur) != cudaSuccess ||
        cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &sdev) != cudaSuccess)
      return GWB_E_LAUNCH;
    if (sdev != cur) return GWB_E_SHAPE;
  }
  unsigned char* base = nullptr;
  rc = noalloc_scratch(&base);
  if (rc) return rc;
  void* a_q8 = base;
  void* a_scale_k8 = base + codes_b;
  void* la = rank_pad ? static_cast<void*>(base + codes_b + scale_b) : nullptr;
  return gwb_svdq_w4a4_linear(x, smooth, proj_down_t, w_q8, w_scale_k8, proj_up, bias, M, N,
                              K, rank_pad, gelu, a_q8, a_scale_k8, la, out, stream);
}
