// noalloc.cu -- ggufmm_gemm_noalloc: the tensor-core GEMM for callers that
// cannot allocate device memory.
//
// ggufmm_gemm needs a scratch workspace (the weight dequantized to fp16 plus
// the activations cast to fp16). Most callers hand one in, but some cannot
// obtain device memory at all at the point of the call: a host that owns
// every byte of the GPU through its own fixed pool and exposes no allocator
// across the FFI, or code that must not allocate once serving has started.
// For them this entry point uses a scratch buffer that lives inside this
// library: a file-scope __device__ array of GGUFMM_NOALLOC_SCRATCH_BYTES.
//
// Facts a caller needs:
//  * The array exists on every GPU that loads this library's device code and
//    stays allocated there until the process exits.
//  * Problems whose scratch (N*K*2 + M*K*2 bytes, each rounded up to 256)
//    exceeds the array are rejected with GGUFMM_ERR_WORKSPACE before anything
//    is launched.
//  * The first call on a device looks up the array's device address (with
//    that device current) and caches it; make that first call before any
//    stream capture.
//  * Every call shares the one array. Calls whose kernels can overlap on the
//    GPU (different streams, or several host threads) race on it and corrupt
//    each other's results; serialise them. Each call fully rewrites the part
//    of the array it reads, so no contents need to start at zero and stale
//    data from an earlier call is never used.
//  * Nothing here calls cudaMalloc, cudaFree or any allocating library
//    routine.
#include <mutex>

#include "common.cuh"

namespace ggufmm {

cudaError_t launch_dequant(const void* q, int qtype, int64_t n_rows, int64_t k, void* out, int out_dtype,
                           cudaStream_t st);
cudaError_t launch_cast_x_f16(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, void* out,
                              cudaStream_t st);
cudaError_t launch_gemm_f16(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k, void* y, int ytype,
                            int64_t ldy, cudaStream_t st, float* part, size_t part_bytes);
int record_cuda_status(cudaError_t e);  // capi.cu: keeps the code for ggufmm_last_cuda_error

// The library-owned scratch. In host code this name is only a stand-in for the
// symbol, not a device address; the address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[GGUFMM_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
cudaError_t scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

int block_weights(int qtype) {
  return (qtype == kQ4_0 || qtype == kQ8_0) ? 32 : (qtype == kQ4_K || qtype == kQ6_K) ? 256 : 0;
}
size_t round256(size_t v) { return (v + 255) / 256 * 256; }
}  // namespace

}  // namespace ggufmm

using namespace ggufmm;

extern "C" int ggufmm_gemm_noalloc(const void* q, int qtype, int64_t n, int64_t k, const void* x, int x_dtype,
                                   int64_t m, int64_t ldx, void* y, int y_dtype, int64_t ldy, void* stream) {
  if (!q || !x || !y) return GGUFMM_ERR_ARG;
  if (!block_weights(qtype)) return GGUFMM_ERR_QTYPE;
  const int xs = x_dtype == GGUFMM_F32 ? 4 : (x_dtype == GGUFMM_F16 || x_dtype == GGUFMM_BF16) ? 2 : 0;
  const int ys = y_dtype == GGUFMM_F32 ? 4 : (y_dtype == GGUFMM_F16 || y_dtype == GGUFMM_BF16) ? 2 : 0;
  if (!xs || !ys) return GGUFMM_ERR_DTYPE;
  if (n <= 0 || k <= 0 || m <= 0 || k % block_weights(qtype) || k > (1 << 20) || n > INT32_MAX || m > INT32_MAX ||
      ldx < k || ldy < n)
    return GGUFMM_ERR_SHAPE;
  const size_t w_bytes = round256(static_cast<size_t>(n) * k * 2);
  const size_t need = w_bytes + round256(static_cast<size_t>(m) * k * 2);
  if (need > GGUFMM_NOALLOC_SCRATCH_BYTES) return GGUFMM_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(q) & 1) || (reinterpret_cast<uintptr_t>(x) & (xs - 1)) ||
      (reinterpret_cast<uintptr_t>(y) & (ys - 1)))
    return GGUFMM_ERR_ALIGN;
  int dev = 0, major = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (e != cudaSuccess) return record_cuda_status(e);
  if (major != 10) return GGUFMM_ERR_DEVICE;
  void* scratch = nullptr;
  e = scratch_address(&scratch);
  if (e != cudaSuccess) return record_cuda_status(e);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* w16 = static_cast<uint8_t*>(scratch);
  uint8_t* x16 = w16 + w_bytes;
  e = launch_dequant(q, qtype, n, k, w16, GGUFMM_F16, st);
  if (e == cudaSuccess) e = launch_cast_x_f16(x, x_dtype, m, k, ldx, x16, st);
  if (e == cudaSuccess) e = launch_gemm_f16(w16, x16, n, m, k, y, y_dtype, ldy, st, nullptr, 0);
  return record_cuda_status(e);
}
