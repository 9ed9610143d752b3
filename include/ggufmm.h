/*
 * ggufmm.h -- C ABI of the B200 (sm_100a) GGUF block-quantized matmul library
 * (libggufmm.so).
 *
 * The library replaces the quantized-matmul dispatch of maci0/vllm-webgpu:
 * the WGSL kernels vllm_webgpu/shaders/generic/matmul_quant.wgsl:20-61
 * (decode GEMV) and matmul_quant_mr4.wgsl:77-131 (multi-row "prefill"), which
 * the models reach through BaseWebGPUModel._dispatch("matmul_quant",
 * [x, W, scales, out], {K, N, USE_QUANT}, ...) (vllm_webgpu/models/base.py:62-100,
 * call sites vllm_webgpu/models/llama.py:276-283,328-332,343-348,355-359).
 * Weights are GGUF blocks exactly as gguf.GGUFReader yields them
 * (vllm_webgpu/quant/gguf_loader.py:137-162): row-major [N, K/block*type_size]
 * bytes, never repacked.
 *
 * Conventions (all entry points):
 *   - every pointer is a caller-owned DEVICE pointer; nothing here allocates
 *     device memory (the GEMM takes an explicit workspace);
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream); work is stream-ordered and no entry point synchronizes;
 *   - the return value is GGUFMM_OK (0) or a negative GGUFMM_ERR_* code.
 *     Argument errors are detected on the host before any launch, so a
 *     failed call enqueues nothing. The reference raised ValueError for bad
 *     shapes (vllm_webgpu/models/llama.py:45-54); the Python binding maps the
 *     codes back to ValueError / RuntimeError;
 *   - entry points are thread-safe and may be called concurrently on
 *     different streams.
 */
#ifndef GGUFMM_H_
#define GGUFMM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GGUFMM_VERSION 100 /* 1.0.0 */

/* Quantization types: the GGMLQuantizationType ids of gguf-py
 * (gguf/constants.py:4059-4073), which GGUFReader reports per tensor. */
enum ggufmm_qtype {
  GGUFMM_Q4_0 = 2,  /* 32 weights / 18 B: fp16 d, 16 B nibbles            */
  GGUFMM_Q8_0 = 8,  /* 32 weights / 34 B: fp16 d, 32 x int8               */
  GGUFMM_Q4_K = 12, /* 256 weights / 144 B: fp16 d,dmin, 12 B 6-bit sc/m, 128 B nibbles */
  GGUFMM_Q6_K = 14  /* 256 weights / 210 B: 128 B ql, 64 B qh, 16 x int8 sc, fp16 d */
};

/* Element types of activations and outputs. */
enum ggufmm_dtype {
  GGUFMM_F32 = 0,
  GGUFMM_F16 = 1,
  GGUFMM_BF16 = 2
};

enum ggufmm_status {
  GGUFMM_OK = 0,
  GGUFMM_ERR_QTYPE = -1,     /* unsupported quantization type            */
  GGUFMM_ERR_SHAPE = -2,     /* K not a multiple of the block, M/N/K <= 0 or too large */
  GGUFMM_ERR_ALIGN = -3,     /* a pointer is not aligned as required      */
  GGUFMM_ERR_DTYPE = -4,     /* unsupported activation / output dtype     */
  GGUFMM_ERR_WORKSPACE = -5, /* workspace NULL or smaller than required   */
  GGUFMM_ERR_CUDA = -6,      /* a CUDA launch or device query failed      */
  GGUFMM_ERR_ARG = -7,       /* NULL pointer or other invalid argument    */
  GGUFMM_ERR_DEVICE = -8     /* the current device is not sm_100          */
};

/* Library version (GGUFMM_VERSION of the build). */
int ggufmm_version(void);

/* Block geometry of a qtype: weights per block / bytes per block; 0 when the
 * qtype is unsupported. Mirrors gguf GGML_QUANT_SIZES (constants.py:4231-4245). */
int ggufmm_block_size(int qtype);
int ggufmm_type_size(int qtype);

/* Human-readable text for a status code (static storage). */
const char* ggufmm_status_string(int status);

/* The last CUDA error code seen by this thread inside the library (0 if none). */
int ggufmm_last_cuda_error(void);

/*
 * Device-side status word: every spin-wait inside the kernels is bounded and,
 * when it gives up, ORs 1 into this word and unwinds instead of hanging; an
 * embedding id out of range ORs 2. Returns the word (>= 0; 0 = nothing seen)
 * or a negative status.
 * Synchronizes `stream`; clears the word when `clear` is nonzero.
 */
int ggufmm_device_status(int clear, void* stream);

/*
 * Poll limit of every bounded wait on the current device (0 restores the
 * default of 2^24 polls, seconds of waiting). A lower limit makes a wait that
 * can never complete -- a peer GPU that never publishes its partials in
 * ggufmm_gemv_allreduce -- give up within milliseconds; tests use it to check
 * that such a call returns, reports the timeout through ggufmm_device_status,
 * and leaves the context usable. Synchronous; call it between launches.
 * No reference counterpart: the reference has no device-side waits.
 */
int ggufmm_set_wait_limit(uint32_t polls);

/*
 * Dequantize `n_rows` rows of `k` weights: out[n, k] (row-major, out_dtype
 * F32 or F16). With out_dtype F32 the result is bit-identical to
 * gguf.quants.dequantize (gguf quants.py:241-251, 396-401, 504-522, 555-572),
 * which is what the reference's loader decodes with
 * (vllm_webgpu/quant/gguf_loader.py:143-159). F16 rounds that fp32 value once
 * (round-to-nearest-even). `q` needs 2-byte alignment, `out` 16-byte.
 */
int ggufmm_dequantize(const void* q, int qtype, int64_t n_rows, int64_t k,
                      void* out, int out_dtype, void* stream);

/*
 * Host <-> device staging by a kernel: copies `bytes` from src to dst, either of
 * which may be page-locked host memory mapped for the device (cudaHostAlloc /
 * torch pin_memory with unified addressing) or device memory. Replaces the
 * reference's buffer upload and staging-buffer readback
 * (vllm_webgpu/webgpu/buffer.py:34, :46-63). Unlike a memcpy, it runs on the SMs
 * and is launched as a programmatic dependent launch, so inside a captured decode
 * step it chains with the GEMV launches (which stream their weights while the
 * activations arrive) instead of handing over to a copy engine. Both pointers
 * 16-byte aligned; pageable host memory gives GGUFMM_ERR_ARG. Stream-ordered.
 */
int ggufmm_stage_copy(void* dst, const void* src, size_t bytes, void* stream);

/*
 * Quantized embedding lookup: out[t, :] = dequantize(row ids[t] of the table) for
 * t < n_ids. Replaces the reference's embedding_lookup dispatch
 * (vllm_webgpu/models/llama.py:170-178, shaders/generic/embedding_lookup.wgsl),
 * which copied rows of an f16 table; here the table stays in its GGUF blocks
 * (token_embd.weight, [n_vocab, k/block*type_size]). out_dtype F32 is
 * bit-identical to gguf.quants.dequantize of the row; F16 / BF16 round that value
 * once. ids are int32 (the reference's u32 token ids below 2^31). An id outside
 * [0, n_vocab) gives a zero row and sets bit 2 of the device status word
 * (ggufmm_device_status). q needs 2-byte alignment, out 16-byte alignment and a
 * row stride ldo (elements, >= k) whose bytes are a multiple of 16.
 */
int ggufmm_embedding(const void* q, int qtype, int64_t n_vocab, int64_t k,
                     const int32_t* ids, int64_t n_ids,
                     void* out, int out_dtype, int64_t ldo, void* stream);

/*
 * Decode GEMV: y[m, n] = sum_k x[m, k] * W[n, k] for 1 <= M <= 8 tokens.
 * Replaces matmul_quant.wgsl:20-61 (one thread per output row there).
 *   q       GGUF blocks [N, K/block*type_size], 16-byte aligned base (rows
 *           need not be 16-byte multiples: Q6_K rows of K = 5120 / 3584 / 1536
 *           are 4200 / 2940 / 1260 bytes)
 *   x       activations [M, K], row stride `ldx` elements (>= K), x_dtype
 *           F32 / F16 / BF16
 *   y       outputs [M, N], row stride `ldy` elements (>= N), y_dtype
 *           F32 / F16 / BF16
 * fp32 accumulation; max|y - y_ref| / rms(y_ref) <= 2e-3 against the fp32
 * dequantize-then-matmul.
 */
int ggufmm_gemv(const void* q, int qtype, int64_t n, int64_t k,
                const void* x, int x_dtype, int64_t m, int64_t ldx,
                void* y, int y_dtype, int64_t ldy, void* stream);

/*
 * Decode GEMV of up to 4 weights that read the same activations, in one
 * launch: y_i[m, n_i] = sum_k x[m, k] W_i[n_i, k], all W_i of one qtype and K.
 * Replaces the separate q/k/v and gate/up dispatches of one layer
 * (vllm_webgpu/models/llama.py:276-283 and 343-348), the way vLLM fuses
 * QKV and gate_up projections. Same requirements and error gate as
 * ggufmm_gemv per weight; falls back to one ggufmm_gemv per weight when the
 * shapes cannot share a launch.
 */
int ggufmm_gemv_grouped(int nseg, const void* const* q, const int64_t* n, int qtype, int64_t k,
                        const void* x, int x_dtype, int64_t m, int64_t ldx,
                        void* const* y, int y_dtype, const int64_t* ldy, void* stream);

/*
 * GEMM of up to 4 weights that read the same activations (q/k/v, gate/up) at
 * any M: y_i[m, n_i] = sum_k x[m, k] W_i[n_i, k], all W_i of one qtype and K.
 * The batched-decode counterpart of ggufmm_gemv_grouped, replacing the same
 * separate dispatches (vllm_webgpu/models/llama.py:276-283 and 343-348) when
 * more than 8 tokens are in flight. workspace: at least
 * ggufmm_gemm_workspace_size(qtype, M, max of n_i, K) bytes, 256-byte aligned.
 * Q4_K at M <= 1024 runs as ONE fused-dequant launch over all the weights' row
 * tiles (the activations cast once); otherwise one ggufmm_gemm per weight.
 */
int ggufmm_gemm_grouped(int nseg, const void* const* q, const int64_t* n, int qtype, int64_t k,
                        const void* x, int x_dtype, int64_t m, int64_t ldx,
                        void* const* y, int y_dtype, const int64_t* ldy,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Decode GEMV with the residual add in its epilogue: y = x W^T + resid for
 * 1 <= M <= 8, Q4_K / Q4_0 with K a multiple of 256 (GGUFMM_ERR_SHAPE /
 * GGUFMM_ERR_QTYPE otherwise, nothing launched). resid has y_dtype and row
 * stride ldr (>= N) and may be y itself (in place). Replaces the o / down
 * projection plus the add shader that follows it (vllm_webgpu/models/llama.py:329-335
 * and 357-363, shaders/generic/add.wgsl): the sum is formed in fp32 and rounded
 * once into y.
 */
int ggufmm_gemv_residual(const void* q, int qtype, int64_t n, int64_t k,
                         const void* x, int x_dtype, int64_t m, int64_t ldx,
                         void* y, int y_dtype, int64_t ldy, const void* resid, int64_t ldr, void* stream);

/*
 * Which decode GEMV kernel ggufmm_gemv would launch for this shape on the
 * current device (nothing is launched): GGUFMM_GEMV_INT8 (integer tensor-core
 * GEMV, Q4_K / Q4_0), GGUFMM_GEMV_F16 (fp16 tensor-core GEMV),
 * GGUFMM_GEMV_STREAM (CUDA-core streaming GEMV, the fallback), or a negative
 * GGUFMM_ERR_* code (GGUFMM_ERR_ALIGN: rows that are not 16-byte multiples and
 * too large for the fp16 GEMV's shared memory, which no decode GEMV stages). The reference dispatches one matmul shader per projection
 * whatever the shape (vllm_webgpu/models/llama.py:276-283); callers use this to
 * send shapes that only the fallback takes to ggufmm_gemm instead.
 */
enum { GGUFMM_GEMV_STREAM = 0, GGUFMM_GEMV_F16 = 1, GGUFMM_GEMV_INT8 = 2 };
int ggufmm_gemv_kernel(int qtype, int64_t n, int64_t k, int64_t m, int x_dtype);

/*
 * Fused SwiGLU decode GEMV: y[m, n] = silu(sum_k x[m, k] Wg[n, k]) * (sum_k x[m, k] Wu[n, k])
 * for 1 <= M <= 8, the gate and up weights (same qtype, N and K) streamed by one
 * launch and combined in its epilogue (silu(g) = g / (1 + exp(-g)), fp32). It
 * replaces the reference's gate and up dispatches (vllm_webgpu/models/llama.py:343-348)
 * plus its SwiGLU shader (shaders/generic/gelu_mul.wgsl:14-20: silu(gate) * up in
 * fp32, dispatched at llama.py:350-352), which the reference runs as three passes. Q4_K and Q4_0 with K a multiple of
 * 256 only (GGUFMM_ERR_QTYPE / GGUFMM_ERR_SHAPE otherwise, nothing launched);
 * the other requirements are those of ggufmm_gemv. Tolerance: the gate and up
 * sums are those of ggufmm_gemv; the product is formed in fp32.
 */
int ggufmm_gemv_swiglu(const void* q_gate, const void* q_up, int qtype, int64_t n, int64_t k,
                       const void* x, int x_dtype, int64_t m, int64_t ldx,
                       void* y, int y_dtype, int64_t ldy, void* stream);

/*
 * Decode GEMV whose result is all-reduced (summed) over `world` GPUs in the same
 * kernel, through NVLink peer memory: the tensor-parallel FFN's / layer's down and o
 * projections (each GPU holds a column slice of W over its share of the inner
 * dimension), replacing the GEMV followed by a separate all-reduce. Every GPU of the
 * group makes this call with the same shapes; each CTA's epilogue stores its fp32
 * partials, each tagged with the call's generation in the same 8-byte word, into every
 * GPU's exchange buffer over NVLink, then polls its own buffer (bounded) until the
 * other GPUs' words of the same rows carry that generation and stores the sum of the
 * partials in rank order, so all GPUs hold bit-identical y[m, n]. The generation is a
 * per-CTA counter kept in the exchange buffer (device memory), so the call can be
 * captured in a CUDA graph and replayed.
 *   peer_bufs  the `world` exchange buffers (device pointers valid on this GPU,
 *              e.g. from CUDA IPC / symmetric memory; 256-byte aligned), each
 *              ggufmm_gemv_allreduce_buffer_bytes(n, m_max, world) bytes and
 *              zero-filled before the first call
 *   epoch      must be nonzero; not used otherwise (kept for compatibility: the
 *              generation lives in device memory)
 * Q4_K / Q4_0, 1 <= M <= m_max <= 8, 2 <= world <= 8; otherwise as ggufmm_gemv.
 * A GPU whose peers never make the matching call gives up after a bounded wait
 * (ggufmm_device_status reports it). The reference has no multi-GPU path.
 */
size_t ggufmm_gemv_allreduce_buffer_bytes(int64_t n, int64_t m_max, int world);
int ggufmm_gemv_allreduce(const void* q, int qtype, int64_t n, int64_t k,
                          const void* x, int x_dtype, int64_t m, int64_t ldx,
                          void* y, int y_dtype, int64_t ldy,
                          void* const* peer_bufs, int world, int rank, int64_t m_max,
                          uint32_t epoch, void* stream);

/*
 * The N-split prefill GEMM with its all-gather in the epilogue: this GPU's column slice
 * W [n, K] of a weight split over `world` GPUs; every output value is stored into all
 * `world` outputs y_peers[i] ([M, ldy], this GPU's and its peers' buffers mapped over
 * NVLink, e.g. symmetric memory) at column col0 + row, so the gather overlaps the MMAs
 * of later tiles instead of following the GEMM. Replaces the GEMM followed by an NCCL
 * all-gather; call ggufmm_peer_barrier afterwards before reading the gathered output.
 * Dequantize + cast + tcgen05 GEMM (workspace: ggufmm_gemm_workspace_size(qtype, M, n, K)).
 * The reference has no multi-GPU path.
 */
int ggufmm_gemm_allgather(const void* q, int qtype, int64_t n, int64_t k,
                          const void* x, int x_dtype, int64_t m, int64_t ldx,
                          void* const* y_peers, int world, int64_t col0, int y_dtype, int64_t ldy,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * One-shot all-reduce (sum) of n <= 65536 fp32 values (n a multiple of 4; in, out and
 * resid 16-byte aligned) over `world` GPUs through NVLink peer memory, for the
 * tensor-parallel decode step's all-reduces (the o / down partials, M x hidden). Every
 * GPU of the group calls it with the same n: each stores its input into every GPU's
 * exchange buffer, raises a per-chunk flag there (generation counters kept in device
 * memory: the call may be captured in a CUDA graph and replayed), waits (bounded) for
 * its own flags and writes out = the sum of all ranks' inputs in rank order (+ resid),
 * the same bits on every GPU. `out` may be `in`.
 *   peer_bufs  the `world` exchange buffers (valid on this GPU, e.g. symmetric memory
 *              or CUDA IPC; 256-byte aligned), ggufmm_allreduce_buffer_bytes(n, world) bytes
 *              each, zero-filled before the first call
 * A peer that never makes the matching call makes the wait give up (bit 1 of
 * ggufmm_device_status) and out is left unwritten. The reference has no multi-GPU path.
 */
size_t ggufmm_allreduce_buffer_bytes(int64_t n, int world);
/* The same kernel with no data (exchange buffers of ggufmm_allreduce_buffer_bytes(0,
 * world) bytes or larger): a barrier across the group's GPUs, after which every rank's earlier work
 * on its stream -- stores into peers' memory included -- is complete and visible. */
int ggufmm_peer_barrier(void* const* peer_bufs, int world, int rank, void* stream);
int ggufmm_allreduce(const float* in, float* out, int64_t n, void* const* peer_bufs, int world, int rank,
                     const float* resid, void* stream);

/*
 * Bytes of workspace ggufmm_gemm uses for this problem on the current device (0
 * for unsupported arguments): the fp16 weight and activations (required; this
 * part grows with M) followed by fp32 partial tiles for the GEMM's tail split
 * (optional: when the workspace is shorter the last wave of tiles runs unsplit).
 * Size it once for the largest M and reuse it.
 */
size_t ggufmm_gemm_workspace_size(int qtype, int64_t m, int64_t n, int64_t k);

/*
 * Prefill / batched GEMM on the sm_100a tensor cores (tcgen05.mma with TMEM
 * accumulators, operands staged by TMA): y[m, n] = sum_k x[m, k] * W[n, k],
 * any M >= 1. Replaces the never-dispatched matmul_quant_mr4.wgsl:77-131
 * (and the token-at-a-time prefill of run_inference.py:323-350). Operands are
 * fp16 (the dequantized fp32 weight rounded once; bf16 activations convert
 * exactly), accumulation fp32. Same layout and error gate as ggufmm_gemv.
 * `workspace` (device, 256-byte aligned) must hold
 * ggufmm_gemm_workspace_size() bytes; its contents are scratch.
 */
int ggufmm_gemm(const void* q, int qtype, int64_t n, int64_t k,
                const void* x, int x_dtype, int64_t m, int64_t ldx,
                void* y, int y_dtype, int64_t ldy,
                void* workspace, size_t workspace_bytes, void* stream);

/*
 * GEMM (any M) with the FFN epilogues, the batched-decode / prefill counterparts of
 * ggufmm_gemv_swiglu and ggufmm_gemv_residual:
 *   ggufmm_gemm_swiglu:   y = silu(x Wg^T) * (x Wu^T)  (gate and up of one qtype, N, K)
 *   ggufmm_gemm_residual: y = x W^T + resid            (resid in y's dtype, stride ldr, may be y)
 * replacing the reference's gate/up dispatches + gelu_mul shader
 * (vllm_webgpu/models/llama.py:343-352, shaders/generic/gelu_mul.wgsl:14-20) and the
 * o / down dispatch + add shader (llama.py:329-335, 355-363). The GEMM leaves fp32
 * partial sums in the workspace (Q4_K at M <= 1024: the fused-dequant kernel, one launch
 * for gate and up; otherwise dequantize + tcgen05 GEMM per weight) and one pass sums
 * them in a fixed order, applies the epilogue in fp32 and rounds once into y.
 * workspace: ggufmm_gemm_ffn_workspace_size(qtype, M, N, K, swiglu) bytes, 256-byte
 * aligned. Same argument gate as ggufmm_gemm.
 */
size_t ggufmm_gemm_ffn_workspace_size(int qtype, int64_t m, int64_t n, int64_t k, int swiglu);
/* The epilogue pass alone, over fp32 sums the caller already has (e.g. from a grouped
 * decode GEMV): swiglu != 0: sums [m, 2n] (gate | up) -> y = silu(gate) * up;
 * swiglu == 0: sums [m, n] -> y = sums + resid. */
int ggufmm_ffn_epilogue(const float* sums, int64_t m, int64_t n, int swiglu, const void* resid, int64_t ldr,
                        void* y, int y_dtype, int64_t ldy, void* stream);
int ggufmm_gemm_swiglu(const void* q_gate, const void* q_up, int qtype, int64_t n, int64_t k,
                       const void* x, int x_dtype, int64_t m, int64_t ldx,
                       void* y, int y_dtype, int64_t ldy,
                       void* workspace, size_t workspace_bytes, void* stream);
int ggufmm_gemm_residual(const void* q, int qtype, int64_t n, int64_t k,
                         const void* x, int x_dtype, int64_t m, int64_t ldx,
                         void* y, int y_dtype, int64_t ldy, const void* resid, int64_t ldr,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * ggufmm_gemm without a caller-provided workspace, for callers that cannot
 * allocate device memory (for example a host whose own pool owns the GPU's
 * memory and offers no allocator across the FFI, or code that must not
 * allocate once it is serving). This entry point has no counterpart in the
 * reference.
 *
 * Its scratch is a library-owned __device__ array of
 * GGUFMM_NOALLOC_SCRATCH_BYTES that every GPU loading the library keeps until
 * the process exits. A problem needing more than that (N*K*2 + M*K*2 bytes,
 * each rounded up to 256) returns GGUFMM_ERR_WORKSPACE and launches nothing.
 * The first call on a device looks up the array's address with that device
 * current; make it before any stream capture. All calls share the array:
 * calls that can overlap on the GPU (other streams, other host threads) race
 * and must be serialised by the caller. No cudaMalloc/cudaFree is made.
 * Same arguments, results and error gate as ggufmm_gemm.
 */
#define GGUFMM_NOALLOC_SCRATCH_BYTES (64u << 20) /* 64 MiB */

int ggufmm_gemm_noalloc(const void* q, int qtype, int64_t n, int64_t k,
                        const void* x, int x_dtype, int64_t m, int64_t ldx,
                        void* y, int y_dtype, int64_t ldy, void* stream);

/*
 * y = x @ W^T choosing the kernel by M (GEMV for M <= 8, GEMM otherwise), the
 * way vLLM's GGUF linear method picks between its GEMV and GEMM kernels
 * (vllm/model_executor/layers/quantization/gguf.py:198-230). The workspace
 * may be NULL when M <= 8.
 */
int ggufmm_mul_mat(const void* q, int qtype, int64_t n, int64_t k,
                   const void* x, int x_dtype, int64_t m, int64_t ldx,
                   void* y, int y_dtype, int64_t ldy,
                   void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GGUFMM_H_ */
