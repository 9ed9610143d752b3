// capi.cu -- the extern "C" boundary of libggufmm (declared in include/ggufmm.h).
//
// Argument validation happens here, on the host, before anything is enqueued:
// a failing call launches nothing and returns a negative status. This mirrors
// the reference's host-side checks (ValueError for bad dimensions in
// vllm_webgpu/models/llama.py:45-54; FileNotFoundError/RuntimeError for a
// missing pipeline in vllm_webgpu/webgpu/pipeline.py:25-30).
#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace ggufmm {

cudaError_t launch_dequant(const void* q, int qtype, int64_t n_rows, int64_t k, void* out, int out_dtype,
                           cudaStream_t st);
cudaError_t launch_cast_x_f16(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, void* out,
                              cudaStream_t st);
cudaError_t launch_gemv(const void* q, int qtype, int64_t n, int64_t k, const void* x, int xtype, int64_t m,
                        int64_t ldx, void* y, int ytype, int64_t ldy, int64_t row_bytes, cudaStream_t st);
cudaError_t gemv_device_error(int* v, int clear, cudaStream_t st);
cudaError_t gemm_fused_device_error(int* v, int clear, cudaStream_t st);
cudaError_t launch_gemm_fused_q4k(const void* q, const void* x16, int64_t n, int64_t m, int64_t k, void* y, int ytype,
                                  int64_t ldy, void* part_ws, size_t part_bytes, cudaStream_t st);
cudaError_t launch_gemm_fused_q4k_grouped(int nseg, const void* const* q, const int64_t* n, const void* x16,
                                          int64_t m, int64_t k, void* const* y, int ytype, const int64_t* ldy,
                                          void* part_ws, size_t part_bytes, cudaStream_t st);
cudaError_t launch_gemm_fused_q4k_partials(int nseg, const void* const* q, const int64_t* n, const void* x16,
                                           int64_t m, int64_t k, void* part_ws, size_t part_bytes, int* zs_out,
                                           cudaStream_t st);
cudaError_t launch_ffn_epilogue(const float* part, int ks, int64_t m, int64_t n, int mode, const void* resid,
                                int64_t ldr, void* y, int ytype, int64_t ldy, cudaStream_t st);
cudaError_t gemv_mma_device_error(int* v, int clear, cudaStream_t st);
bool gemv_mma_supported(int qtype, int64_t n, int64_t k, int m, int xtype);
cudaError_t launch_gemv_mma_grouped(int nseg, const void* const* q, const int64_t* n, int qtype, int64_t k,
                                    const void* x, int xtype, int64_t m, int64_t ldx, void* const* y, int ytype,
                                    const int64_t* ldy, int64_t row_bytes, cudaStream_t st);
cudaError_t launch_gemv_mma(const void* q, int qtype, int64_t n, int64_t k, const void* x, int xtype, int64_t m,
                            int64_t ldx, void* y, int ytype, int64_t ldy, int64_t row_bytes, cudaStream_t st);
cudaError_t gemm_device_error(int* v, int clear, cudaStream_t st);
cudaError_t gemv_i8_device_error(int* v, int clear, cudaStream_t st);
cudaError_t dequant_device_error(int* v, int clear, cudaStream_t st);
cudaError_t launch_embedding(const void* q, int qtype, int64_t n_vocab, int64_t k, const int32_t* ids, int64_t n_ids,
                             void* out, int out_dtype, int64_t ldo, cudaStream_t st);
cudaError_t gemv_set_wait_limit(uint32_t polls);
size_t allreduce_buffer_bytes(int64_t n, int world);
cudaError_t launch_allreduce_oneshot(const float* in, float* out, int64_t n, void* const* bufs, int world, int rank,
                                     const void* resid, cudaStream_t st);
cudaError_t allreduce_device_error(int* v, int clear, cudaStream_t st);
cudaError_t launch_gemm_f16_peers(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k,
                                  void* const* ys, int world, int64_t col0, int ytype, int64_t ldy, cudaStream_t st,
                                  float* part, size_t part_bytes);
cudaError_t allreduce_set_wait_limit(uint32_t polls);
cudaError_t gemm_set_wait_limit(uint32_t polls);
cudaError_t gemv_mma_set_wait_limit(uint32_t polls);
cudaError_t gemm_fused_set_wait_limit(uint32_t polls);
cudaError_t gemv_i8_set_wait_limit(uint32_t polls);
bool gemv_i8_supported(int qtype, int64_t k, int m);
cudaError_t launch_gemv_i8_grouped(int nseg, const void* const* q, const int64_t* n, int qtype, int64_t k,
                                   const void* x, int xtype, int64_t m, int64_t ldx, void* const* y, int ytype,
                                   const int64_t* ldy, int64_t row_bytes, cudaStream_t st, int swiglu,
                                   const struct GemvTp* tp, const void* resid = nullptr, int64_t ldr = 0);
struct GemvTp {
  int world, rank;
  uint32_t epoch;
  int64_t m_max;
  const void* const* bufs;
};
size_t gemv_tp_buffer_bytes(int64_t n, int64_t m_max, int world);
cudaError_t launch_gemm_f16(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k, void* y, int ytype,
                            int64_t ldy, cudaStream_t st, float* part, size_t part_bytes);
size_t gemm_tail_bytes(int64_t n, int64_t m, int64_t k);

struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
};

static constexpr int kMaxDev = 64;
static DevInfo g_dev[kMaxDev];
static std::once_flag g_dev_once[kMaxDev];
static int g_dev_major[kMaxDev];

DevInfo device_info(int dev) {
  if (dev < 0 || dev >= kMaxDev) return DevInfo{};
  std::call_once(g_dev_once[dev], [dev] {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) g_dev[dev].sms = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess)
      g_dev[dev].smem_optin = v;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess) g_dev_major[dev] = v;
  });
  return g_dev[dev];
}

static thread_local int t_last_cuda_error = 0;

static int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return GGUFMM_OK;
  t_last_cuda_error = static_cast<int>(e);
  return GGUFMM_ERR_CUDA;
}

// For entry points defined in other translation units: records the CUDA error
// (read back by ggufmm_last_cuda_error) and maps it to a status.
int record_cuda_status(cudaError_t e) { return cuda_status(e); }

static int check_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  device_info(dev);
  if (dev >= kMaxDev || g_dev_major[dev] != 10) return GGUFMM_ERR_DEVICE;
  return GGUFMM_OK;
}

static int block_of(int qtype) {
  switch (qtype) {
    case kQ4_0: case kQ8_0: return 32;
    case kQ4_K: case kQ6_K: return 256;
    default: return 0;
  }
}
static int bytes_of(int qtype) {
  switch (qtype) {
    case kQ4_0: return 18;
    case kQ8_0: return 34;
    case kQ4_K: return 144;
    case kQ6_K: return 210;
    default: return 0;
  }
}
static int elem_size(int dtype) {
  switch (dtype) {
    case GGUFMM_F32: return 4;
    case GGUFMM_F16: case GGUFMM_BF16: return 2;
    default: return 0;
  }
}
static bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

static constexpr int64_t kMaxK = 1 << 20;

static int check_matmul_args(const void* q, int qtype, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m,
                             int64_t ldx, const void* y, int y_dtype, int64_t ldy) {
  if (!q || !x || !y) return GGUFMM_ERR_ARG;
  if (!block_of(qtype)) return GGUFMM_ERR_QTYPE;
  if (!elem_size(x_dtype) || !elem_size(y_dtype)) return GGUFMM_ERR_DTYPE;
  if (n <= 0 || k <= 0 || m <= 0 || k > kMaxK || n > (int64_t(1) << 31) - 1 || m > (int64_t(1) << 31) - 1)
    return GGUFMM_ERR_SHAPE;
  if (k % block_of(qtype)) return GGUFMM_ERR_SHAPE;
  if (ldx < k || ldy < n) return GGUFMM_ERR_SHAPE;
  return GGUFMM_OK;
}

}  // namespace ggufmm

using namespace ggufmm;

extern "C" {

int ggufmm_version(void) { return GGUFMM_VERSION; }
int ggufmm_block_size(int qtype) { return block_of(qtype); }
int ggufmm_type_size(int qtype) { return bytes_of(qtype); }
int ggufmm_last_cuda_error(void) { return t_last_cuda_error; }

const char* ggufmm_status_string(int s) {
  switch (s) {
    case GGUFMM_OK: return "ok";
    case GGUFMM_ERR_QTYPE: return "unsupported quantization type";
    case GGUFMM_ERR_SHAPE: return "invalid shape (K must be a multiple of the block size; M, N, K > 0; ld >= row length)";
    case GGUFMM_ERR_ALIGN: return "misaligned pointer or row stride";
    case GGUFMM_ERR_DTYPE: return "unsupported dtype";
    case GGUFMM_ERR_WORKSPACE: return "workspace missing or too small";
    case GGUFMM_ERR_CUDA: return "CUDA error";
    case GGUFMM_ERR_ARG: return "invalid argument";
    case GGUFMM_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    default: return "unknown status";
  }
}

int ggufmm_device_status(int clear, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int a = 0, b = 0, c = 0, d = 0, f = 0, h = 0;
  cudaError_t e = gemv_device_error(&a, clear, st);
  if (e == cudaSuccess) e = gemm_device_error(&b, clear, st);
  if (e == cudaSuccess) e = gemv_mma_device_error(&c, clear, st);
  if (e == cudaSuccess) e = gemm_fused_device_error(&d, clear, st);
  if (e == cudaSuccess) e = gemv_i8_device_error(&f, clear, st);
  if (e == cudaSuccess) e = dequant_device_error(&h, clear, st);
  int r = 0;
  if (e == cudaSuccess) e = allreduce_device_error(&r, clear, st);
  if (e != cudaSuccess) return cuda_status(e);
  return a | b | c | d | f | h | r;
}

int ggufmm_set_wait_limit(uint32_t polls) {
  const uint32_t v = polls ? polls : (1u << 24);
  cudaError_t e = gemv_set_wait_limit(v);
  if (e == cudaSuccess) e = gemm_set_wait_limit(v);
  if (e == cudaSuccess) e = gemv_mma_set_wait_limit(v);
  if (e == cudaSuccess) e = gemm_fused_set_wait_limit(v);
  if (e == cudaSuccess) e = gemv_i8_set_wait_limit(v);
  if (e == cudaSuccess) e = allreduce_set_wait_limit(v);
  return cuda_status(e);
}

size_t ggufmm_allreduce_buffer_bytes(int64_t n, int world) { return allreduce_buffer_bytes(n, world); }

int ggufmm_allreduce(const float* in, float* out, int64_t n, void* const* peer_bufs, int world, int rank,
                     const float* resid, void* stream) {
  if (!in || !out || !peer_bufs) return GGUFMM_ERR_ARG;
  if (world < 2 || world > 8 || rank < 0 || rank >= world) return GGUFMM_ERR_ARG;
  if (n <= 0 || !allreduce_buffer_bytes(n, world)) return GGUFMM_ERR_SHAPE;
  if (!aligned(in, 16) || !aligned(out, 16) || (resid && !aligned(resid, 16))) return GGUFMM_ERR_ALIGN;
  for (int i = 0; i < world; ++i)
    if (!peer_bufs[i] || !aligned(peer_bufs[i], 256)) return GGUFMM_ERR_ALIGN;
  if (!aligned(in, 4) || !aligned(out, 4) || (resid && !aligned(resid, 4))) return GGUFMM_ERR_ALIGN;
  int s = check_device();
  if (s) return s;
  return cuda_status(launch_allreduce_oneshot(in, out, n, peer_bufs, world, rank, resid,
                                              static_cast<cudaStream_t>(stream)));
}

int ggufmm_peer_barrier(void* const* peer_bufs, int world, int rank, void* stream) {
  if (!peer_bufs || world < 2 || world > 8 || rank < 0 || rank >= world) return GGUFMM_ERR_ARG;
  for (int i = 0; i < world; ++i)
    if (!peer_bufs[i] || !aligned(peer_bufs[i], 256)) return GGUFMM_ERR_ALIGN;
  int s = check_device();
  if (s) return s;
  return cuda_status(launch_allreduce_oneshot(nullptr, nullptr, 0, peer_bufs, world, rank, nullptr,
                                              static_cast<cudaStream_t>(stream)));
}

int ggufmm_dequantize(const void* q, int qtype, int64_t n_rows, int64_t k, void* out, int out_dtype, void* stream) {
  if (!q || !out) return GGUFMM_ERR_ARG;
  if (!block_of(qtype)) return GGUFMM_ERR_QTYPE;
  if (out_dtype != GGUFMM_F32 && out_dtype != GGUFMM_F16) return GGUFMM_ERR_DTYPE;
  if (n_rows <= 0 || k <= 0 || k % block_of(qtype) || k > kMaxK) return GGUFMM_ERR_SHAPE;
  if (!aligned(q, 2) || !aligned(out, 16)) return GGUFMM_ERR_ALIGN;
  int s = check_device();
  if (s) return s;
  return cuda_status(launch_dequant(q, qtype, n_rows, k, out, out_dtype, static_cast<cudaStream_t>(stream)));
}

int ggufmm_embedding(const void* q, int qtype, int64_t n_vocab, int64_t k, const int32_t* ids, int64_t n_ids,
                     void* out, int out_dtype, int64_t ldo, void* stream) {
  if (!q || !ids || !out) return GGUFMM_ERR_ARG;
  if (!block_of(qtype)) return GGUFMM_ERR_QTYPE;
  if (!elem_size(out_dtype)) return GGUFMM_ERR_DTYPE;
  if (n_vocab <= 0 || n_ids <= 0 || k <= 0 || k % block_of(qtype) || k > kMaxK || ldo < k ||
      n_ids > (int64_t(1) << 31) - 1)
    return GGUFMM_ERR_SHAPE;
  if (!aligned(q, 2) || !aligned(ids, 4) || !aligned(out, 16) || (ldo * elem_size(out_dtype)) % 16)
    return GGUFMM_ERR_ALIGN;
  int s = check_device();
  if (s) return s;
  return cuda_status(launch_embedding(q, qtype, n_vocab, k, ids, n_ids, out, out_dtype, ldo,
                                      static_cast<cudaStream_t>(stream)));
}

int ggufmm_gemv(const void* q, int qtype, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m, int64_t ldx,
                void* y, int y_dtype, int64_t ldy, void* stream) {
  int s = check_matmul_args(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy);
  if (s) return s;
  if (m > 8) return GGUFMM_ERR_SHAPE;
  const int64_t row_bytes = k / block_of(qtype) * bytes_of(qtype);
  if (!aligned(q, 16) || !aligned(x, 16) || (ldx * elem_size(x_dtype)) % 16 || !aligned(y, elem_size(y_dtype)))
    return GGUFMM_ERR_ALIGN;
  if (row_bytes > 160 * 1024) return GGUFMM_ERR_SHAPE;  // one weight row must fit a shared-memory stage
  s = check_device();
  if (s) return s;
  // Rows that are not 16-byte multiples (Q6_K with K/256 not a multiple of 8, e.g.
  // K = 5120 / 3584 / 1536) are staged by the fp16 tensor-core GEMV only.
  if (row_bytes % 16) {
    if (!gemv_mma_supported(qtype, n, k, static_cast<int>(m), x_dtype)) return GGUFMM_ERR_ALIGN;
    return cuda_status(launch_gemv_mma(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy, row_bytes,
                                       static_cast<cudaStream_t>(stream)));
  }
  // integer tensor-core GEMV (Q4_K, Q4_0), else the fp16 tensor-core GEMV when the
  // shape allows (K a multiple of 256, activations fit in shared memory), else the
  // CUDA-core streaming GEMV
  if (gemv_i8_supported(qtype, k, static_cast<int>(m)))
    return cuda_status(launch_gemv_i8_grouped(1, &q, &n, qtype, k, x, x_dtype, m, ldx, &y, y_dtype, &ldy, row_bytes,
                                              static_cast<cudaStream_t>(stream), 0, nullptr));
  if (gemv_mma_supported(qtype, n, k, static_cast<int>(m), x_dtype))
    return cuda_status(launch_gemv_mma(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy, row_bytes,
                                       static_cast<cudaStream_t>(stream)));
  return cuda_status(launch_gemv(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy, row_bytes,
                                 static_cast<cudaStream_t>(stream)));
}

int ggufmm_gemv_grouped(int nseg, const void* const* q, const int64_t* n, int qtype, int64_t k, const void* x,
                        int x_dtype, int64_t m, int64_t ldx, void* const* y, int y_dtype, const int64_t* ldy,
                        void* stream) {
  if (!q || !n || !y || !ldy) return GGUFMM_ERR_ARG;
  if (nseg < 1 || nseg > 4) return GGUFMM_ERR_SHAPE;
  for (int i = 0; i < nseg; ++i) {
    const int s = check_matmul_args(q[i], qtype, n[i], k, x, x_dtype, m, ldx, y[i], y_dtype, ldy[i]);
    if (s) return s;
  }
  if (m > 8) return GGUFMM_ERR_SHAPE;
  const int64_t row_bytes = k / block_of(qtype) * bytes_of(qtype);
  bool one_launch = row_bytes % 16 == 0 && aligned(x, 16) && (ldx * elem_size(x_dtype)) % 16 == 0;
  for (int i = 0; i < nseg; ++i) one_launch = one_launch && aligned(q[i], 16) && aligned(y[i], elem_size(y_dtype));
  int s = check_device();
  if (s) return s;
  if (one_launch && gemv_i8_supported(qtype, k, static_cast<int>(m)))
    return cuda_status(launch_gemv_i8_grouped(nseg, q, n, qtype, k, x, x_dtype, m, ldx, y, y_dtype, ldy, row_bytes,
                                              static_cast<cudaStream_t>(stream), 0, nullptr));
  if (one_launch && gemv_mma_supported(qtype, n[0], k, static_cast<int>(m), x_dtype))
    return cuda_status(launch_gemv_mma_grouped(nseg, q, n, qtype, k, x, x_dtype, m, ldx, y, y_dtype, ldy, row_bytes,
                                               static_cast<cudaStream_t>(stream)));
  for (int i = 0; i < nseg; ++i) {  // one GEMV per weight
    s = ggufmm_gemv(q[i], qtype, n[i], k, x, x_dtype, m, ldx, y[i], y_dtype, ldy[i], stream);
    if (s) return s;
  }
  return GGUFMM_OK;
}

int ggufmm_gemv_kernel(int qtype, int64_t n, int64_t k, int64_t m, int x_dtype) {
  if (block_of(qtype) == 0) return GGUFMM_ERR_QTYPE;
  if (n <= 0 || k <= 0 || m < 1 || m > 8 || k % block_of(qtype)) return GGUFMM_ERR_SHAPE;
  if (elem_size(x_dtype) == 0) return GGUFMM_ERR_DTYPE;
  const int s = check_device();
  if (s) return s;
  const int64_t row_bytes = k / block_of(qtype) * bytes_of(qtype);
  if (row_bytes % 16 == 0 && gemv_i8_supported(qtype, k, static_cast<int>(m))) return GGUFMM_GEMV_INT8;
  if (gemv_mma_supported(qtype, n, k, static_cast<int>(m), x_dtype)) return GGUFMM_GEMV_F16;
  return row_bytes % 16 ? static_cast<int>(GGUFMM_ERR_ALIGN) : static_cast<int>(GGUFMM_GEMV_STREAM);
}

int ggufmm_gemv_swiglu(const void* q_gate, const void* q_up, int qtype, int64_t n, int64_t k, const void* x,
                       int x_dtype, int64_t m, int64_t ldx, void* y, int y_dtype, int64_t ldy, void* stream) {
  int s = check_matmul_args(q_gate, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy);
  if (s) return s;
  if (!q_up) return GGUFMM_ERR_ARG;
  if (m > 8) return GGUFMM_ERR_SHAPE;
  const int64_t row_bytes = k / block_of(qtype) * bytes_of(qtype);
  if (!aligned(q_gate, 16) || !aligned(q_up, 16) || row_bytes % 16 || !aligned(x, 16) ||
      (ldx * elem_size(x_dtype)) % 16 || !aligned(y, elem_size(y_dtype)))
    return GGUFMM_ERR_ALIGN;
  s = check_device();
  if (s) return s;
  // the fused epilogue lives in the integer tensor-core GEMV (Q4_K, Q4_0, K a multiple of 256)
  if (!gemv_i8_supported(qtype, k, static_cast<int>(m))) return qtype == GGUFMM_Q4_K || qtype == GGUFMM_Q4_0
                                                                    ? GGUFMM_ERR_SHAPE
                                                                    : GGUFMM_ERR_QTYPE;
  const void* qs[2] = {q_gate, q_up};
  const int64_t ns[2] = {n, n};
  void* ys[2] = {y, y};
  const int64_t lds[2] = {ldy, ldy};
  return cuda_status(launch_gemv_i8_grouped(2, qs, ns, qtype, k, x, x_dtype, m, ldx, ys, y_dtype, lds, row_bytes,
                                            static_cast<cudaStream_t>(stream), 1, nullptr));
}

size_t ggufmm_gemv_allreduce_buffer_bytes(int64_t n, int64_t m_max, int world) {
  if (n <= 0 || m_max < 1 || m_max > 8 || world < 2 || world > 8) return 0;
  return gemv_tp_buffer_bytes(n, m_max, world);
}

int ggufmm_gemv_allreduce(const void* q, int qtype, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m,
                          int64_t ldx, void* y, int y_dtype, int64_t ldy, void* const* peer_bufs, int world,
                          int rank, int64_t m_max, uint32_t epoch, void* stream) {
  int s = check_matmul_args(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy);
  if (s) return s;
  if (!peer_bufs) return GGUFMM_ERR_ARG;
  if (world < 2 || world > 8 || rank < 0 || rank >= world || m > m_max || m_max > 8 || epoch == 0)
    return GGUFMM_ERR_ARG;
  for (int i = 0; i < world; ++i)
    if (!peer_bufs[i] || !aligned(peer_bufs[i], 256)) return GGUFMM_ERR_ALIGN;
  const int64_t row_bytes = k / block_of(qtype) * bytes_of(qtype);
  if (!aligned(q, 16) || row_bytes % 16 || !aligned(x, 16) || (ldx * elem_size(x_dtype)) % 16 ||
      !aligned(y, elem_size(y_dtype)))
    return GGUFMM_ERR_ALIGN;
  s = check_device();
  if (s) return s;
  if (!gemv_i8_supported(qtype, k, static_cast<int>(m)))
    return qtype == GGUFMM_Q4_K || qtype == GGUFMM_Q4_0 ? GGUFMM_ERR_SHAPE : GGUFMM_ERR_QTYPE;
  const GemvTp tp{world, rank, epoch, m_max, peer_bufs};
  return cuda_status(launch_gemv_i8_grouped(1, &q, &n, qtype, k, x, x_dtype, m, ldx, &y, y_dtype, &ldy, row_bytes,
                                            static_cast<cudaStream_t>(stream), 0, &tp));
}

int ggufmm_gemv_residual(const void* q, int qtype, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m,
                         int64_t ldx, void* y, int y_dtype, int64_t ldy, const void* resid, int64_t ldr, void* stream) {
  int s = check_matmul_args(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy);
  if (s) return s;
  if (!resid) return GGUFMM_ERR_ARG;
  if (m > 8 || ldr < n) return GGUFMM_ERR_SHAPE;
  const int64_t row_bytes = k / block_of(qtype) * bytes_of(qtype);
  if (!aligned(q, 16) || row_bytes % 16 || !aligned(x, 16) || (ldx * elem_size(x_dtype)) % 16 ||
      !aligned(y, elem_size(y_dtype)) || !aligned(resid, elem_size(y_dtype)))
    return GGUFMM_ERR_ALIGN;
  s = check_device();
  if (s) return s;
  if (!gemv_i8_supported(qtype, k, static_cast<int>(m)))
    return qtype == GGUFMM_Q4_K || qtype == GGUFMM_Q4_0 ? GGUFMM_ERR_SHAPE : GGUFMM_ERR_QTYPE;
  return cuda_status(launch_gemv_i8_grouped(1, &q, &n, qtype, k, x, x_dtype, m, ldx, &y, y_dtype, &ldy, row_bytes,
                                            static_cast<cudaStream_t>(stream), 0, nullptr, resid, ldr));
}

static size_t round256(size_t v) { return (v + 255) / 256 * 256; }

// GGUFMM_GEMM_FUSED=0 selects the two-pass (dequantize, then GEMM) path for Q4_K too.
static bool fused_gemm_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GGUFMM_GEMM_FUSED");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Largest M served by the fused-dequant GEMM (GGUFMM_GEMM_FUSED_MAXM). Above it the
// two-pass path wins: it dequantizes each weight once, the fused GEMM once per
// 256-token tile (measured, Q4_K 14336 x 4096: M = 512 57.6 vs 94.2 us, M = 2048 equal,
// M = 8192 0.886 vs 0.812 ms).
static int64_t fused_gemm_max_m() {
  static const int64_t v = [] {
    const char* e = std::getenv("GGUFMM_GEMM_FUSED_MAXM");
    return e && e[0] ? static_cast<int64_t>(std::atoll(e)) : static_cast<int64_t>(1024);
  }();
  return v;
}

// Two-pass GEMM workspace: [fp16 weight][fp16 activations][fp32 partials of the
// GEMM's tail split]. The first two are required; the GEMM splits its last wave
// along K only when the workspace also holds the third.
static size_t gemm_ws_required(int64_t m, int64_t n, int64_t k) {
  return round256(static_cast<size_t>(n) * k * 2) + round256(static_cast<size_t>(m) * k * 2);
}
size_t ggufmm_gemm_workspace_size(int qtype, int64_t m, int64_t n, int64_t k) {
  if (!block_of(qtype) || m <= 0 || n <= 0 || k <= 0 || k % block_of(qtype)) return 0;
  return gemm_ws_required(m, n, k) + round256(gemm_tail_bytes(n, m, k));
}
// The tail-split region of a two-pass workspace (null when it does not fit).
static float* gemm_tail_region(void* workspace, size_t workspace_bytes, int64_t m, int64_t n, int64_t k,
                               size_t* bytes) {
  const size_t req = gemm_ws_required(m, n, k), tail = gemm_tail_bytes(n, m, k);
  *bytes = 0;
  if (tail == 0 || workspace_bytes < req + tail) return nullptr;
  *bytes = workspace_bytes - req;
  return reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + req);
}

int ggufmm_gemm(const void* q, int qtype, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m, int64_t ldx,
                void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_matmul_args(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy);
  if (s) return s;
  if (!workspace || workspace_bytes < gemm_ws_required(m, n, k)) return GGUFMM_ERR_WORKSPACE;
  if (!aligned(q, 2) || !aligned(workspace, 256) || !aligned(y, elem_size(y_dtype)) ||
      !aligned(x, elem_size(x_dtype)))
    return GGUFMM_ERR_ALIGN;
  s = check_device();
  if (s) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (qtype == kQ4_K && m <= fused_gemm_max_m() && aligned(q, 16) && fused_gemm_enabled()) {
    // dequantization fused into the tensor-core GEMM: only the fp16 activations need
    // scratch (and the K split's partials). Above fused_gemm_max_m() the two-pass path,
    // which dequantizes each weight once instead of once per token tile, is faster.
    cudaError_t e = launch_cast_x_f16(x, x_dtype, m, k, ldx, workspace, st);
    // the K split's fp32 partials go where the two-pass path keeps the fp16 weight
    const size_t x16_bytes = round256(static_cast<size_t>(m) * k * 2);
    if (e == cudaSuccess)
      e = launch_gemm_fused_q4k(q, workspace, n, m, k, y, y_dtype, ldy, static_cast<uint8_t*>(workspace) + x16_bytes,
                                workspace_bytes - x16_bytes, st);
    return cuda_status(e);
  }
  uint8_t* w16 = static_cast<uint8_t*>(workspace);
  uint8_t* x16 = w16 + round256(static_cast<size_t>(n) * k * 2);
  cudaError_t e = launch_dequant(q, qtype, n, k, w16, GGUFMM_F16, st);
  if (e == cudaSuccess) e = launch_cast_x_f16(x, x_dtype, m, k, ldx, x16, st);
  size_t tail_bytes = 0;
  float* tail = gemm_tail_region(workspace, workspace_bytes, m, n, k, &tail_bytes);
  if (e == cudaSuccess) e = launch_gemm_f16(w16, x16, n, m, k, y, y_dtype, ldy, st, tail, tail_bytes);
  return cuda_status(e);
}

int ggufmm_gemm_grouped(int nseg, const void* const* q, const int64_t* n, int qtype, int64_t k, const void* x,
                        int x_dtype, int64_t m, int64_t ldx, void* const* y, int y_dtype, const int64_t* ldy,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (!q || !n || !y || !ldy) return GGUFMM_ERR_ARG;
  if (nseg < 1 || nseg > 4) return GGUFMM_ERR_SHAPE;
  int64_t nmax = 0;
  bool fused = qtype == kQ4_K && m <= fused_gemm_max_m() && fused_gemm_enabled();
  for (int i = 0; i < nseg; ++i) {
    const int s = check_matmul_args(q[i], qtype, n[i], k, x, x_dtype, m, ldx, y[i], y_dtype, ldy[i]);
    if (s) return s;
    nmax = std::max(nmax, n[i]);
    fused = fused && aligned(q[i], 16);
  }
  if (!workspace || workspace_bytes < gemm_ws_required(m, nmax, k)) return GGUFMM_ERR_WORKSPACE;
  if (!aligned(workspace, 256) || !aligned(x, elem_size(x_dtype))) return GGUFMM_ERR_ALIGN;
  for (int i = 0; i < nseg; ++i)
    if (!aligned(q[i], 2) || !aligned(y[i], elem_size(y_dtype))) return GGUFMM_ERR_ALIGN;
  int s = check_device();
  if (s) return s;
  if (!fused) {  // one GEMM per weight, sharing the workspace
    for (int i = 0; i < nseg; ++i) {
      s = ggufmm_gemm(q[i], qtype, n[i], k, x, x_dtype, m, ldx, y[i], y_dtype, ldy[i], workspace, workspace_bytes,
                      stream);
      if (s) return s;
    }
    return GGUFMM_OK;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t x16_bytes = round256(static_cast<size_t>(m) * k * 2);
  cudaError_t e = launch_cast_x_f16(x, x_dtype, m, k, ldx, workspace, st);
  if (e == cudaSuccess)
    e = launch_gemm_fused_q4k_grouped(nseg, q, n, workspace, m, k, y, y_dtype, ldy,
                                      static_cast<uint8_t*>(workspace) + x16_bytes, workspace_bytes - x16_bytes, st);
  return cuda_status(e);
}

// ---- GEMM with the FFN epilogues (SwiGLU of gate and up, residual add) ----------------
// Workspace: [x cast to fp16][fp32 partials, up to 4 K slices x m x (2n | n)][one fp16
// dequantized weight for the two-pass path].
static size_t ffn_x16_bytes(int64_t m, int64_t k) { return round256(static_cast<size_t>(m) * k * 2); }
static size_t ffn_part_bytes(int64_t m, int64_t ntot) { return round256(static_cast<size_t>(4) * m * ntot * 4); }

size_t ggufmm_gemm_ffn_workspace_size(int qtype, int64_t m, int64_t n, int64_t k, int swiglu) {
  if (!block_of(qtype) || m <= 0 || n <= 0 || k <= 0 || k % block_of(qtype)) return 0;
  const int64_t ntot = swiglu ? 2 * n : n;
  return ffn_x16_bytes(m, k) + ffn_part_bytes(m, ntot) + round256(static_cast<size_t>(n) * k * 2);
}

// gate / up (nseg 2, SwiGLU) or one weight (residual): the GEMM into fp32 partials,
// then the epilogue pass into y.
static int gemm_ffn(int nseg, const void* const* qs, int qtype, int64_t n, int64_t k, const void* x, int x_dtype,
                    int64_t m, int64_t ldx, void* y, int y_dtype, int64_t ldy, const void* resid, int64_t ldr,
                    void* workspace, size_t workspace_bytes, void* stream) {
  const size_t need = ggufmm_gemm_ffn_workspace_size(qtype, m, n, k, nseg == 2);
  if (!workspace || workspace_bytes < need) return GGUFMM_ERR_WORKSPACE;
  if (!aligned(workspace, 256) || !aligned(y, elem_size(y_dtype)) || !aligned(x, elem_size(x_dtype)))
    return GGUFMM_ERR_ALIGN;
  for (int i = 0; i < nseg; ++i)
    if (!aligned(qs[i], 2)) return GGUFMM_ERR_ALIGN;
  if (resid && !aligned(resid, elem_size(y_dtype))) return GGUFMM_ERR_ALIGN;
  int s = check_device();
  if (s) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t ntot = nseg * n;
  uint8_t* x16 = static_cast<uint8_t*>(workspace);
  uint8_t* part = x16 + ffn_x16_bytes(m, k);
  const size_t part_bytes = ffn_part_bytes(m, ntot);
  uint8_t* w16 = part + part_bytes;
  cudaError_t e = launch_cast_x_f16(x, x_dtype, m, k, ldx, x16, st);
  int zs = 1;
  bool fused = qtype == kQ4_K && m <= fused_gemm_max_m() && fused_gemm_enabled();
  for (int i = 0; i < nseg; ++i) fused = fused && aligned(qs[i], 16);
  if (e == cudaSuccess && fused) {
    const int64_t ns[2] = {n, n};
    e = launch_gemm_fused_q4k_partials(nseg, qs, ns, x16, m, k, part, part_bytes, &zs, st);
  } else {
    for (int i = 0; i < nseg && e == cudaSuccess; ++i) {  // dequantize -> fp16, tcgen05 GEMM into fp32 columns
      e = launch_dequant(qs[i], qtype, n, k, w16, GGUFMM_F16, st);
      if (e == cudaSuccess)
        e = launch_gemm_f16(w16, x16, n, m, k, reinterpret_cast<float*>(part) + i * n, GGUFMM_F32, ntot, st, nullptr,
                            0);
    }
  }
  if (e == cudaSuccess)
    e = launch_ffn_epilogue(reinterpret_cast<const float*>(part), zs, m, n, nseg == 2 ? 0 : 1, resid, ldr, y, y_dtype,
                            ldy, st);
  return cuda_status(e);
}

int ggufmm_ffn_epilogue(const float* sums, int64_t m, int64_t n, int swiglu, const void* resid, int64_t ldr, void* y,
                        int y_dtype, int64_t ldy, void* stream) {
  if (!sums || !y || (!swiglu && !resid)) return GGUFMM_ERR_ARG;
  if (!elem_size(y_dtype)) return GGUFMM_ERR_DTYPE;
  if (m <= 0 || n <= 0 || ldy < n || (!swiglu && ldr < n)) return GGUFMM_ERR_SHAPE;
  if (!aligned(sums, 4) || !aligned(y, elem_size(y_dtype)) || (resid && !aligned(resid, elem_size(y_dtype))))
    return GGUFMM_ERR_ALIGN;
  int s = check_device();
  if (s) return s;
  return cuda_status(launch_ffn_epilogue(sums, 1, m, n, swiglu ? 0 : 1, resid, ldr, y, y_dtype, ldy,
                                         static_cast<cudaStream_t>(stream)));
}

int ggufmm_gemm_swiglu(const void* q_gate, const void* q_up, int qtype, int64_t n, int64_t k, const void* x,
                       int x_dtype, int64_t m, int64_t ldx, void* y, int y_dtype, int64_t ldy, void* workspace,
                       size_t workspace_bytes, void* stream) {
  int s = check_matmul_args(q_gate, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy);
  if (s) return s;
  if (!q_up) return GGUFMM_ERR_ARG;
  const void* qs[2] = {q_gate, q_up};
  return gemm_ffn(2, qs, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy, nullptr, 0, workspace, workspace_bytes,
                  stream);
}

int ggufmm_gemm_residual(const void* q, int qtype, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m,
                         int64_t ldx, void* y, int y_dtype, int64_t ldy, const void* resid, int64_t ldr,
                         void* workspace, size_t workspace_bytes, void* stream) {
  int s = check_matmul_args(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy);
  if (s) return s;
  if (!resid) return GGUFMM_ERR_ARG;
  if (ldr < n) return GGUFMM_ERR_SHAPE;
  return gemm_ffn(1, &q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy, resid, ldr, workspace, workspace_bytes,
                  stream);
}

int ggufmm_gemm_allgather(const void* q, int qtype, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m,
                          int64_t ldx, void* const* y_peers, int world, int64_t col0, int y_dtype, int64_t ldy,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (!y_peers || world < 1 || world > 8) return GGUFMM_ERR_ARG;
  int s = check_matmul_args(q, qtype, n, k, x, x_dtype, m, ldx, y_peers[0], y_dtype, ldy);
  if (s) return s;
  if (col0 < 0 || col0 + n > ldy) return GGUFMM_ERR_SHAPE;
  if (!workspace || workspace_bytes < gemm_ws_required(m, n, k)) return GGUFMM_ERR_WORKSPACE;
  if (!aligned(q, 2) || !aligned(workspace, 256) || !aligned(x, elem_size(x_dtype))) return GGUFMM_ERR_ALIGN;
  for (int i = 0; i < world; ++i)
    if (!y_peers[i] || !aligned(y_peers[i], elem_size(y_dtype))) return GGUFMM_ERR_ALIGN;
  s = check_device();
  if (s) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* w16 = static_cast<uint8_t*>(workspace);
  uint8_t* x16 = w16 + round256(static_cast<size_t>(n) * k * 2);
  cudaError_t e = launch_dequant(q, qtype, n, k, w16, GGUFMM_F16, st);
  if (e == cudaSuccess) e = launch_cast_x_f16(x, x_dtype, m, k, ldx, x16, st);
  size_t tail_bytes = 0;
  float* tail = gemm_tail_region(workspace, workspace_bytes, m, n, k, &tail_bytes);
  if (e == cudaSuccess)
    e = launch_gemm_f16_peers(w16, x16, n, m, k, y_peers, world, col0, y_dtype, ldy, st, tail, tail_bytes);
  return cuda_status(e);
}

int ggufmm_mul_mat(const void* q, int qtype, int64_t n, int64_t k, const void* x, int x_dtype, int64_t m,
                   int64_t ldx, void* y, int y_dtype, int64_t ldy, void* workspace, size_t workspace_bytes,
                   void* stream) {
  int s = check_matmul_args(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy);
  if (s) return s;
  const int64_t row_bytes = k / block_of(qtype) * bytes_of(qtype);
  const bool gemv_ok = m <= 8 && aligned(q, 16) && row_bytes <= 160 * 1024 && aligned(x, 16) &&
                       (ldx * elem_size(x_dtype)) % 16 == 0 && ggufmm_gemv_kernel(qtype, n, k, m, x_dtype) >= 0;
  // Q4_K shapes that only the streaming GEMV fits run faster on the fused-dequant GEMM,
  // when the caller passed a workspace for it
  const bool gemm_better = qtype == kQ4_K && workspace &&
                           workspace_bytes >= gemm_ws_required(m, n, k) &&
                           ggufmm_gemv_kernel(qtype, n, k, m, x_dtype) == GGUFMM_GEMV_STREAM;
  if (gemv_ok && !gemm_better)
    return ggufmm_gemv(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy, stream);
  return ggufmm_gemm(q, qtype, n, k, x, x_dtype, m, ldx, y, y_dtype, ldy, workspace, workspace_bytes, stream);
}

}  // extern "C"
