// dequant.cu -- GGUF block dequantization on the GPU, bit-identical to
// gguf-py's numpy dequantizers (gguf quants.py:241-251 Q4_0, 396-401 Q8_0,
// 504-522 Q4_K, 555-572 Q6_K), plus the fp16 activation cast the tensor-core
// GEMM consumes.
//
// One thread produces 32 consecutive output weights (one Q4_0/Q8_0 block, one
// Q4_K sub-block, one 32-wide group of a Q6_K superblock). Every product and
// difference is a separately rounded fp32 op (__fmul_rn / __fsub_rn), in the
// order gguf-py evaluates them, so no FMA contraction can change a bit.
// The kernel is HBM-bound on the output write (4 B per weight for fp32).
#include "common.cuh"

namespace ggufmm {

// Load `NW` 32-bit words starting at a 2-byte-aligned global address: aligned
// 32-bit loads (16-byte vector loads when the address allows) and a funnel shift.
// Only words that hold requested bytes are touched.
template <int NW>
__device__ __forceinline__ void ldg_words_a2(const uint8_t* p, uint32_t* w) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if (NW % 4 == 0 && (a & 15) == 0) {
    const uint4* v = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < NW / 4; ++i) {
      const uint4 t = __ldg(v + i);
      w[4 * i] = t.x; w[4 * i + 1] = t.y; w[4 * i + 2] = t.z; w[4 * i + 3] = t.w;
    }
    return;
  }
  const uint32_t* q = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  if ((a & 3) == 0) {
#pragma unroll
    for (int i = 0; i < NW; ++i) w[i] = __ldg(q + i);
    return;
  }
  uint32_t t[NW + 1];
#pragma unroll
  for (int i = 0; i <= NW; ++i) t[i] = __ldg(q + i);
#pragma unroll
  for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(t[i], t[i + 1], 16);
}

// Quants become exact floats without the quarter-rate int->float conversion: a
// byte permute builds the float 2^23 + u from a byte u (bytes u, 0, 0, 0x4B), and
// one subtraction removes the offset (and the format's bias) exactly.

__device__ __forceinline__ uint32_t byte_of(const uint32_t* w, int i) { return (w[i >> 2] >> (8 * (i & 3))) & 0xFFu; }

template <int QT>
__device__ __forceinline__ void dequant32(const uint8_t* row, int unit, float* out);

// Q4_0: d * (nib - 8); byte j: low nibble = elt j, high nibble = elt j+16.
template <>
__device__ __forceinline__ void dequant32<kQ4_0>(const uint8_t* row, int unit, float* o) {
  const uint8_t* b = row + 18 * unit;
  float d = half_bits_to_float(__ldg(reinterpret_cast<const uint16_t*>(b)));
  uint32_t w[4];
  ldg_words_a2<4>(b + 2, w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // bytes q, 0, 0, 0x4B = the float 2^23 + q; minus 2^23 + 8 gives q - 8 exactly
    const uint32_t lo = w[i] & 0x0F0F0F0Fu, hi = (w[i] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      o[4 * i + e] = __fmul_rn(d, __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540u | e)) - 8388616.f);
      o[16 + 4 * i + e] = __fmul_rn(d, __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540u | e)) - 8388616.f);
    }
  }
}

// Q8_0: q * d.
template <>
__device__ __forceinline__ void dequant32<kQ8_0>(const uint8_t* row, int unit, float* o) {
  const uint8_t* b = row + 34 * unit;
  float d = half_bits_to_float(__ldg(reinterpret_cast<const uint16_t*>(b)));
  uint32_t w[8];
  ldg_words_a2<8>(b + 2, w);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // q ^ 0x80 = q + 128 as an unsigned byte: float 2^23 + q + 128, minus 2^23 + 128
    const uint32_t u = w[i] ^ 0x80808080u;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o[4 * i + e] = __fmul_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540u | e)) - 8388736.f, d);
  }
}

// Q4_K sub-block j of superblock sb: (d*sc_j)*q - (dmin*m_j).
__device__ __forceinline__ void q4k_scale_min(const uint32_t* s, int j, uint32_t& sc, uint32_t& m) {
  // s = the 12 scale bytes as 3 little-endian words (bytes 4..15 of the block)
  if (j < 4) {
    sc = byte_of(s, j) & 63u;
    m = byte_of(s, j + 4) & 63u;
  } else {
    sc = (byte_of(s, j + 4) & 15u) | ((byte_of(s, j - 4) >> 6) << 4);
    m = (byte_of(s, j + 4) >> 4) | ((byte_of(s, j) >> 6) << 4);
  }
}

template <>
__device__ __forceinline__ void dequant32<kQ4_K>(const uint8_t* row, int unit, float* o) {
  const int sb = unit >> 3, j = unit & 7;
  const uint8_t* b = row + 144 * sb;
  uint32_t hdr[4];
  ldg_words_a2<4>(b, hdr);  // d, dmin, 12 scale bytes
  float d = half_bits_to_float(hdr[0]);
  float dmin = half_bits_to_float(hdr[0] >> 16);
  uint32_t sc, m;
  q4k_scale_min(hdr + 1, j, sc, m);
  const float dsc = __fmul_rn(d, static_cast<float>(sc));
  const float dm = __fmul_rn(dmin, static_cast<float>(m));
  uint32_t w[8];
  ldg_words_a2<8>(b + 16 + 32 * (j >> 1), w);
  const int sh = 4 * (j & 1);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // four nibbles at once; each becomes the float 2^23 + q with one byte permute
    // (bytes q, 0, 0, 0x4B), minus 2^23 exactly
    const uint32_t nib = (w[i] >> sh) & 0x0F0F0F0Fu;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float qf = __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7540u | e)) - 8388608.f;
      o[4 * i + e] = __fsub_rn(__fmul_rn(dsc, qf), dm);
    }
  }
}

// Q6_K group g (0..7) of superblock sb: element e = 32g + c, h = g/4, u = g%4:
//   q6 = ((ql[h*64 + (u%2)*32 + c] >> 4*(u/2)) & 15) | (((qh[h*32 + c] >> 2u) & 3) << 4)
//   value = (d * sc[e/16]) * (q6 - 32)
template <>
__device__ __forceinline__ void dequant32<kQ6_K>(const uint8_t* row, int unit, float* o) {
  const int sb = unit >> 3, g = unit & 7, h = g >> 2, u = g & 3;
  const uint8_t* b = row + 210 * sb;
  uint32_t ql[8], qh[8];
  ldg_words_a2<8>(b + h * 64 + (u & 1) * 32, ql);
  ldg_words_a2<8>(b + 128 + h * 32, qh);
  const uint16_t scw = __ldg(reinterpret_cast<const uint16_t*>(b + 192 + 2 * g));
  const float d = half_bits_to_float(__ldg(reinterpret_cast<const uint16_t*>(b + 208)));
  const float dl0 = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(scw & 0xFF)));
  const float dl1 = __fmul_rn(d, static_cast<float>(static_cast<int8_t>(scw >> 8)));
  const int shl = 4 * (u >> 1), shh = 2 * u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // four 6-bit quants per word: low nibble | 2 high bits << 4; float 2^23 + q6, minus 2^23 + 32
    const uint32_t q6 = ((ql[i] >> shl) & 0x0F0F0F0Fu) | (((qh[i] >> shh) & 0x03030303u) << 4);
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o[4 * i + e] = __fmul_rn(i < 4 ? dl0 : dl1, __uint_as_float(__byte_perm(q6, 0x4B000000u, 0x7540u | e)) - 8388640.f);
  }
}

// The 32 outputs of a lane are staged in shared memory (XOR-swizzled 16-byte
// slots, conflict-free) so that every global store instruction of a warp writes
// 512 contiguous bytes.
template <int QT, int OT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ q, int64_t n_units,
                                                      int units_per_row, int64_t row_bytes,
                                                      void* __restrict__ out) {
  constexpr int kChunks = OT == GGUFMM_F32 ? 8 : 4;  // 16-byte chunks per lane (32 outputs)
  __shared__ uint4 stage[8][32 * kChunks];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t warp_u0 = u - lane;
  uint4* st = stage[wid];
  if (u < n_units) {
    const int64_t r = u / units_per_row;
    const int c = static_cast<int>(u - r * units_per_row);
    float v[32];
    dequant32<QT>(q + r * row_bytes, c, v);
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
      uint4 w;
      if (OT == GGUFMM_F32) {
        w = make_uint4(__float_as_uint(v[4 * i]), __float_as_uint(v[4 * i + 1]), __float_as_uint(v[4 * i + 2]),
                       __float_as_uint(v[4 * i + 3]));
      } else {
        uint32_t h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __half2 h2 = __floats2half2_rn(v[8 * i + 2 * j], v[8 * i + 2 * j + 1]);
          h[j] = *reinterpret_cast<uint32_t*>(&h2);
        }
        w = make_uint4(h[0], h[1], h[2], h[3]);
      }
      st[lane * kChunks + (i ^ (lane & (kChunks - 1)))] = w;
    }
  }
  __syncwarp();
  uint4* o = reinterpret_cast<uint4*>(static_cast<uint8_t*>(out)) + warp_u0 * kChunks;
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    const int gi = j * 32 + lane;  // 16-byte chunk index within the warp's output range
    const int src = gi / kChunks, ch = gi % kChunks;
    if (warp_u0 + src < n_units) o[gi] = st[src * kChunks + (ch ^ (src & (kChunks - 1)))];
  }
}

template <int QT, int OT>
static cudaError_t launch_dequant_t(const void* q, int64_t n_rows, int64_t k, void* out, cudaStream_t st) {
  const int64_t units_per_row = k / 32;
  const int64_t n_units = n_rows * units_per_row;
  const int64_t row_bytes = k / QTraits<QT>::kBlock * QTraits<QT>::kBytes;
  const int threads = 256;
  const int64_t blocks = (n_units + threads - 1) / threads;
  dequant_kernel<QT, OT><<<static_cast<unsigned>(blocks), threads, 0, st>>>(
      static_cast<const uint8_t*>(q), n_units, static_cast<int>(units_per_row), row_bytes, out);
  return cudaGetLastError();
}

cudaError_t launch_dequant(const void* q, int qtype, int64_t n_rows, int64_t k, void* out, int out_dtype,
                           cudaStream_t st) {
#define GGUFMM_DQ(QT)                                                                     \
  case QT:                                                                                \
    return out_dtype == GGUFMM_F32 ? launch_dequant_t<QT, GGUFMM_F32>(q, n_rows, k, out, st) \
                                   : launch_dequant_t<QT, GGUFMM_F16>(q, n_rows, k, out, st);
  switch (qtype) {
    GGUFMM_DQ(kQ4_0)
    GGUFMM_DQ(kQ8_0)
    GGUFMM_DQ(kQ4_K)
    GGUFMM_DQ(kQ6_K)
    default:
      return cudaErrorInvalidValue;
  }
#undef GGUFMM_DQ
}

// ---- quantized embedding lookup ------------------------------------------------------
// out[t, :] = dequantize(table row ids[t]) for t < n_ids: the reference's
// embedding_lookup shader (vllm_webgpu/shaders/generic/embedding_lookup.wgsl, one
// workgroup per token copying an f16 row), on the GGUF blocks of the table itself
// (token_embd is usually Q4_K / Q6_K in a GGUF file). One thread per 32 outputs, the
// same bit-exact decode as dequant_kernel; fp32 output is gguf's value, f16 / bf16 its
// single rounding. An id outside [0, n_vocab) writes a zero row and sets
// kErrIndex in the device status word (the reference does not check).
constexpr int kErrIndex = 2;

template <int OT>
__device__ __forceinline__ void store32(void* out, const float* v) {
  uint4* o = reinterpret_cast<uint4*>(out);
  if (OT == GGUFMM_F32) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      o[i] = make_uint4(__float_as_uint(v[4 * i]), __float_as_uint(v[4 * i + 1]), __float_as_uint(v[4 * i + 2]),
                        __float_as_uint(v[4 * i + 3]));
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = v[8 * i + 2 * j], b = v[8 * i + 2 * j + 1];
        if (OT == GGUFMM_F16) {
          __half2 h2 = __floats2half2_rn(a, b);
          h[j] = *reinterpret_cast<uint32_t*>(&h2);
        } else {
          __nv_bfloat162 h2 = __floats2bfloat162_rn(a, b);
          h[j] = *reinterpret_cast<uint32_t*>(&h2);
        }
      }
      o[i] = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
}

template <int QT, int OT>
__global__ void __launch_bounds__(256) embed_kernel(const uint8_t* __restrict__ q, int64_t n_vocab, int64_t row_bytes,
                                                    int units_per_row, const int32_t* __restrict__ ids, int64_t n_ids,
                                                    void* __restrict__ out, int64_t ldo) {
  const int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (u >= n_ids * units_per_row) return;
  const int64_t t = u / units_per_row;
  const int c = static_cast<int>(u - t * units_per_row);
  const int64_t id = __ldg(ids + t);
  float v[32];
  if (id >= 0 && id < n_vocab) {
    dequant32<QT>(q + id * row_bytes, c, v);
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = 0.f;
    if (c == 0) atomicOr(&g_device_error, kErrIndex);
  }
  constexpr int es = OT == GGUFMM_F32 ? 4 : 2;
  store32<OT>(static_cast<uint8_t*>(out) + (t * ldo + 32 * c) * es, v);
}

template <int QT, int OT>
static cudaError_t launch_embed_t(const void* q, int64_t n_vocab, int64_t k, const int32_t* ids, int64_t n_ids,
                                  void* out, int64_t ldo, cudaStream_t st) {
  const int units_per_row = static_cast<int>(k / 32);
  const int64_t n_units = n_ids * units_per_row;
  const int64_t row_bytes = k / QTraits<QT>::kBlock * QTraits<QT>::kBytes;
  const int threads = 256;
  embed_kernel<QT, OT><<<static_cast<unsigned>((n_units + threads - 1) / threads), threads, 0, st>>>(
      static_cast<const uint8_t*>(q), n_vocab, row_bytes, units_per_row, ids, n_ids, out, ldo);
  return cudaGetLastError();
}

cudaError_t launch_embedding(const void* q, int qtype, int64_t n_vocab, int64_t k, const int32_t* ids, int64_t n_ids,
                             void* out, int out_dtype, int64_t ldo, cudaStream_t st) {
#define GGUFMM_EMB(QT)                                                                                   \
  case QT:                                                                                               \
    return out_dtype == GGUFMM_F32   ? launch_embed_t<QT, GGUFMM_F32>(q, n_vocab, k, ids, n_ids, out, ldo, st) \
           : out_dtype == GGUFMM_F16 ? launch_embed_t<QT, GGUFMM_F16>(q, n_vocab, k, ids, n_ids, out, ldo, st) \
                                     : launch_embed_t<QT, GGUFMM_BF16>(q, n_vocab, k, ids, n_ids, out, ldo, st);
  switch (qtype) {
    GGUFMM_EMB(kQ4_0)
    GGUFMM_EMB(kQ8_0)
    GGUFMM_EMB(kQ4_K)
    GGUFMM_EMB(kQ6_K)
    default:
      return cudaErrorInvalidValue;
  }
#undef GGUFMM_EMB
}

cudaError_t dequant_device_error(int* v, int clear, cudaStream_t st) { return tu_device_error(v, clear, st); }

// Activation cast x[M, K] (row stride ldx, f32/f16/bf16) -> fp16 [M, K]
// contiguous, 8 elements per thread. bf16 -> fp16 is exact for |x| in the
// fp16 normal range; values beyond +-65504 become +-inf.
// Any alignment: element loads.
template <int XT>
__global__ void __launch_bounds__(256) cast_x_f16_scalar_kernel(const void* __restrict__ x, int64_t m, int64_t k,
                                                         int64_t ldx, __half* __restrict__ out) {
  // the next kernel (the GEMM) may start its read-only weight stream now; this one
  // waits for its predecessor: x may come from it, out may still be read by it
  pdl_trigger();
  pdl_wait();
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  const int64_t total = m * k;
  if (i >= total) return;
  const int64_t r = i / k, c = i - r * k;
  __half tmp[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (c + j < k) {
      float v;
      if (XT == GGUFMM_F32) v = static_cast<const float*>(x)[r * ldx + c + j];
      else if (XT == GGUFMM_F16) v = __half2float(static_cast<const __half*>(x)[r * ldx + c + j]);
      else v = __bfloat162float(static_cast<const __nv_bfloat16*>(x)[r * ldx + c + j]);
      tmp[j] = __float2half_rn(v);
    } else {
      tmp[j] = __float2half_rn(0.f);
    }
  }
  // k is a multiple of 32, so c..c+7 never straddles a row and out+i is 16-byte aligned.
  *reinterpret_cast<uint4*>(out + i) = *reinterpret_cast<uint4*>(tmp);
}

// 16-byte aligned rows: vector loads (fp16 input is a plain copy).
template <int XT>
__global__ void __launch_bounds__(256) cast_x_f16_kernel(const void* __restrict__ x, int64_t m, int64_t k,
                                                         int64_t ldx, __half* __restrict__ out) {
  // the next kernel (the GEMM) may start its read-only weight stream now; this one
  // waits for its predecessor: x may come from it, out may still be read by it
  pdl_trigger();
  pdl_wait();
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  const int64_t total = m * k;
  if (i >= total) return;
  const int64_t r = i / k, c = i - r * k;
  // k is a multiple of 32, so c..c+7 never straddles a row and out+i is 16-byte aligned;
  // the caller guarantees 16-byte aligned input rows (row stride and base)
  float v[8];
  if (XT == GGUFMM_F32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + r * ldx + c);
    const float4 a = p[0], b = p[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 p = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + r * ldx + c);
    if (XT == GGUFMM_F16) {
      *reinterpret_cast<uint4*>(out + i) = p;
      return;
    }
    const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[2 * j] = __uint_as_float(w[j] << 16);
      v[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  }
  uint32_t h[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    __half2 h2 = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
    h[j] = *reinterpret_cast<uint32_t*>(&h2);
  }
  *reinterpret_cast<uint4*>(out + i) = make_uint4(h[0], h[1], h[2], h[3]);
}

cudaError_t launch_cast_x_f16(const void* x, int x_dtype, int64_t m, int64_t k, int64_t ldx, void* out,
                              cudaStream_t st) {
  const int64_t n8 = (m * k + 7) / 8;
  const unsigned blocks = static_cast<unsigned>((n8 + 255) / 256);
  __half* o = static_cast<__half*>(out);
  const int es = x_dtype == GGUFMM_F32 ? 4 : 2;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (ldx * es) % 16 == 0;
  // programmatic dependent launch: the kernel waits for its predecessor before touching
  // memory, and the GEMM after it may start its weight stream while it runs
  void (*fn)(const void*, int64_t, int64_t, int64_t, __half*);
  if (vec)
    fn = x_dtype == GGUFMM_F32 ? cast_x_f16_kernel<GGUFMM_F32>
         : x_dtype == GGUFMM_F16 ? cast_x_f16_kernel<GGUFMM_F16> : cast_x_f16_kernel<GGUFMM_BF16>;
  else
    fn = x_dtype == GGUFMM_F32 ? cast_x_f16_scalar_kernel<GGUFMM_F32>
         : x_dtype == GGUFMM_F16 ? cast_x_f16_scalar_kernel<GGUFMM_F16> : cast_x_f16_scalar_kernel<GGUFMM_BF16>;
  return pdl_launch(fn, dim3(blocks), dim3(256), 0, st, x, m, k, ldx, o);
}

}  // namespace ggufmm
