// gemv.cu -- decode GEMV over GGUF blocks, y[m, n] = sum_k x[m, k] W[n, k],
// for M <= 8 tokens. Replaces matmul_quant.wgsl:20-61 of maci0/vllm-webgpu
// (one thread per output row walking K byte by byte, never vectorised).
//
// Design (HBM-bound; the weights are read exactly once):
//  * A CTA owns row tiles of kRows consecutive weight rows. Rows of one tile
//    are contiguous in memory, so one elected thread streams a whole tile
//    into a shared-memory stage with a single 1-D bulk TMA copy
//    (cp.async.bulk, completion on an mbarrier). `stages` tiles are in flight
//    per CTA; no registers are spent on loads in flight.
//  * Every thread owns fixed 32-weight "segments" of K (one Q4_0/Q8_0 block,
//    16 bytes of a Q4_K nibble chunk, one 32-group of a Q6_K superblock) and
//    keeps the matching activations in registers (fp32) across all tiles.
//  * Integer quants are turned into floats without a conversion instruction:
//    the quant is OR-ed into the mantissa of 1.0f, giving 1 + q*2^-s exactly;
//    sum x*(1+q*2^-s) - sum x = 2^-s * sum q*x (the cancellation loses < 2^-17
//    of the dot product). Products run on the packed fp32x2 FMA of sm_100.
//  * GGUF scales are applied once per sub-block to the integer dot products,
//    so per weight the inner loop is ~1 shift + 1 mask + 1/2 FFMA2.
//  * Per-row partial sums are reduced with warp shuffles, then across warps in
//    shared memory; fp32 throughout.
#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace ggufmm {

constexpr int kRows = 4;  // weight rows per stage

struct GemvArgs {
  const uint8_t* q;
  int64_t n;
  int64_t row_bytes;
  const void* x;
  int64_t ldx;
  void* y;
  int64_t ldy;
  int xtype;
  int ytype;
  int nseg;       // K / 32
  int stages;     // smem stages per CTA
  int rows;       // weight rows per tile (1..kRows; fewer when rows are wide)
  int64_t ntiles; // ceil(N / rows)
  uint32_t stage_bytes;
};

// ---- segment geometry ------------------------------------------------------
// Each segment covers 32 weights whose activations are two runs of 16:
// x[k0 .. k0+15] and x[k1 .. k1+15].
template <int QT>
__device__ __forceinline__ void seg_k(int seg, int& k0, int& k1) {
  if (QT == kQ4_K) {
    const int sb = seg >> 3, p = seg & 7;
    k0 = 256 * sb + 64 * (p >> 1) + 16 * (p & 1);
    k1 = k0 + 32;
  } else if (QT == kQ6_K) {
    k0 = 32 * seg;  // group g = seg&7 of superblock seg>>3 covers 32 contiguous weights
    k1 = k0 + 16;
  } else {
    k0 = 32 * seg;
    k1 = k0 + 16;
  }
}

// ---- shared-memory byte access ----------------------------------------------
// Load NW words from byte offset `off` (2-byte aligned) of a word array.
template <int NW>
__device__ __forceinline__ void lds_words_a2(const uint32_t* base, uint32_t off, uint32_t* w) {
  const uint32_t* p = base + (off >> 2);
  const uint32_t sh = (off & 3u) * 8u;
  uint32_t t[NW + 1];
#pragma unroll
  for (int i = 0; i <= NW; ++i) t[i] = p[i];
#pragma unroll
  for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(t[i], t[i + 1], sh);
}

__device__ __forceinline__ uint32_t lds_u16(const uint32_t* base, uint32_t off) {
  return (base[off >> 2] >> ((off & 2u) * 8u)) & 0xFFFFu;
}

// Move byte B of w to bits 15..22 (low nibble -> 15..18, high nibble -> 19..22).
template <int B>
__device__ __forceinline__ uint32_t byte_to_15(uint32_t w) {
  if (B == 0) return w << 15;
  if (B == 1) return w << 7;
  if (B == 2) return w >> 1;
  return w >> 9;
}

constexpr uint32_t kOne = 0x3F800000u;

// Packed fp32x2 FMA (sm_100 FFMA2), or two scalar FMAs when
// GGUFMM_GEMV_SCALAR_FMA is defined (kept for A/B instruction-count checks).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
#ifdef GGUFMM_GEMV_SCALAR_FMA
  return make_float2(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y));
#else
  return __ffma2_rn(a, b, c);
#endif
}

__device__ __forceinline__ float2 f2bits(uint32_t a, uint32_t b) {
  return make_float2(__uint_as_float(a), __uint_as_float(b));
}

// acc += {1 + lo(b)*2^-8 ..} . xl and {1 + hi(b)*2^-4 ..} . xh for the 8 nibbles
// of w; xl[0] = x of bytes (0,1), xl[1] = x of bytes (2,3) (same for xh).
__device__ __forceinline__ void nib_word_dot(uint32_t w, const float2* xl, const float2* xh, float2& al,
                                             float2& ah) {
  const uint32_t s0 = byte_to_15<0>(w), s1 = byte_to_15<1>(w), s2 = byte_to_15<2>(w), s3 = byte_to_15<3>(w);
  al = fma2(f2bits((s0 & 0x00078000u) | kOne, (s1 & 0x00078000u) | kOne), xl[0], al);
  al = fma2(f2bits((s2 & 0x00078000u) | kOne, (s3 & 0x00078000u) | kOne), xl[1], al);
  ah = fma2(f2bits((s0 & 0x00780000u) | kOne, (s1 & 0x00780000u) | kOne), xh[0], ah);
  ah = fma2(f2bits((s2 & 0x00780000u) | kOne, (s3 & 0x00780000u) | kOne), xh[1], ah);
}

// Per-token activation state for one segment: v[i] = (x[slot 2i], x[slot 2i+1]),
// slots 0..15 = x[k0..k0+15], slots 16..31 = x[k1..k1+15].
struct XSeg {
  float2 v[16];
  float s0, s1;  // sums of the two halves
};

__device__ __forceinline__ void load_xseg(const void* x, int xtype, int64_t row_off, int k0, int k1, XSeg& xs) {
  float t[32];
  if (xtype == GGUFMM_BF16) {
    load_x16<GGUFMM_BF16>(x, row_off + k0, t);
    load_x16<GGUFMM_BF16>(x, row_off + k1, t + 16);
  } else if (xtype == GGUFMM_F16) {
    load_x16<GGUFMM_F16>(x, row_off + k0, t);
    load_x16<GGUFMM_F16>(x, row_off + k1, t + 16);
  } else {
    load_x16<GGUFMM_F32>(x, row_off + k0, t);
    load_x16<GGUFMM_F32>(x, row_off + k1, t + 16);
  }
  float a = 0.f, b = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    a += t[i];
    b += t[16 + i];
  }
#pragma unroll
  for (int i = 0; i < 16; ++i) xs.v[i] = make_float2(t[2 * i], t[2 * i + 1]);
  xs.s0 = a;
  xs.s1 = b;
}

// ---- per-format segment dot products ------------------------------------------
// `base` = stage words, `row` = byte offset of the weight row inside the stage.
// Computes out[m] += sum over the segment of x[m, k] * W[row, k] for NT tokens.
template <int QT, int NT>
__device__ __forceinline__ void seg_dot(const uint32_t* base, uint32_t row, int seg, const XSeg* xs, float* out);

// Q4_K: segment p of superblock sb = 16 bytes of nibble chunk c = p/2 (half p&1);
// low nibbles belong to sub-block 2c, high nibbles to sub-block 2c+1.
template <int NT>
__device__ __forceinline__ void seg_dot_q4k(const uint32_t* base, uint32_t row, int seg, const XSeg* xs,
                                            float* out) {
  const int sb = seg >> 3, p = seg & 7, c = p >> 1;
  const uint32_t blk = row + 144u * sb;  // 16-byte aligned
  const uint4 hdr = *reinterpret_cast<const uint4*>(base + (blk >> 2));
  const uint4 qv = *reinterpret_cast<const uint4*>(base + ((blk + 16u + 32u * c + 16u * (p & 1)) >> 2));
  const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
  // 6-bit scales/mins (gguf quants.py:479-501), four sub-blocks per word, branch-free:
  //   sub-blocks 0..3: sc = s[j] & 63,  m = s[j+4] & 63
  //   sub-blocks 4..7: sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4,  m = (s[j+4] >> 4) | (s[j] >> 6) << 4
  const uint32_t scw = c < 2 ? (hdr.y & 0x3F3F3F3Fu) : ((hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u));
  const uint32_t mw = c < 2 ? (hdr.z & 0x3F3F3F3Fu) : (((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u));
  const uint32_t sh = 16u * (c & 1);  // sub-blocks 2c, 2c+1 are bytes (2c&3), (2c&3)+1 of the word
  const float dsc0 = d * static_cast<float>((scw >> sh) & 0xFFu) * 256.f;
  const float dsc1 = d * static_cast<float>((scw >> (sh + 8)) & 0xFFu) * 16.f;
  const float dm0 = dmin * static_cast<float>((mw >> sh) & 0xFFu);
  const float dm1 = dmin * static_cast<float>((mw >> (sh + 8)) & 0xFFu);
  const uint32_t w[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float2 al = make_float2(-xs[t].s0, 0.f), ah = make_float2(-xs[t].s1, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) nib_word_dot(w[i], xs[t].v + 2 * i, xs[t].v + 8 + 2 * i, al, ah);
    // al = 2^-8 sum q_lo x, ah = 2^-4 sum q_hi x
    out[t] += dsc0 * (al.x + al.y) - dm0 * xs[t].s0 + dsc1 * (ah.x + ah.y) - dm1 * xs[t].s1;
  }
}

// Q4_0: block = fp16 d + 16 bytes; byte j low nibble -> x[k0+j], high -> x[k0+16+j];
// value d*(q-8).
template <int NT>
__device__ __forceinline__ void seg_dot_q40(const uint32_t* base, uint32_t row, int seg, const XSeg* xs,
                                            float* out) {
  const uint32_t blk = row + 18u * seg;
  const float d = half_bits_to_float(lds_u16(base, blk));
  uint32_t w[4];
  lds_words_a2<4>(base, blk + 2u, w);
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float2 al = make_float2(-xs[t].s0, 0.f), ah = make_float2(-xs[t].s1, 0.f);
#pragma unroll
    for (int i = 0; i < 4; ++i) nib_word_dot(w[i], xs[t].v + 2 * i, xs[t].v + 8 + 2 * i, al, ah);
    const float qx = 256.f * (al.x + al.y) + 16.f * (ah.x + ah.y);
    out[t] += d * (qx - 8.f * (xs[t].s0 + xs[t].s1));
  }
}

// Q8_0: block = fp16 d + 32 x int8; q+128 is OR-ed into the mantissa as 1 + u*2^-8.
template <int NT>
__device__ __forceinline__ void seg_dot_q80(const uint32_t* base, uint32_t row, int seg, const XSeg* xs,
                                            float* out) {
  const uint32_t blk = row + 34u * seg;
  const float d = half_bits_to_float(lds_u16(base, blk));
  uint32_t w[8];
  lds_words_a2<8>(base, blk + 2u, w);
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] ^= 0x80808080u;  // int8 q -> u8 q+128
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float2 a = make_float2(-(xs[t].s0 + xs[t].s1), 0.f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t s0 = byte_to_15<0>(w[i]), s1 = byte_to_15<1>(w[i]), s2 = byte_to_15<2>(w[i]),
                     s3 = byte_to_15<3>(w[i]);
      a = fma2(f2bits((s0 & 0x007F8000u) | kOne, (s1 & 0x007F8000u) | kOne), xs[t].v[2 * i], a);
      a = fma2(f2bits((s2 & 0x007F8000u) | kOne, (s3 & 0x007F8000u) | kOne), xs[t].v[2 * i + 1], a);
    }
    out[t] += d * (256.f * (a.x + a.y) - 128.f * (xs[t].s0 + xs[t].s1));
  }
}

// Q6_K: group g of superblock sb; q6 (6 bits) is OR-ed into the mantissa as
// 1 + q6*2^-6; value (d*sc)*(q6-32) with one int8 scale per 16 weights.
template <int NT>
__device__ __forceinline__ void seg_dot_q6k(const uint32_t* base, uint32_t row, int seg, const XSeg* xs,
                                            float* out) {
  const int sb = seg >> 3, g = seg & 7, h = g >> 2, u = g & 3;
  const uint32_t blk = row + 210u * sb;
  uint32_t ql[8], qh[8];
  lds_words_a2<8>(base, blk + 64u * h + 32u * (u & 1), ql);
  lds_words_a2<8>(base, blk + 128u + 32u * h, qh);
  const uint32_t scw = lds_u16(base, blk + 192u + 2u * g);
  const float d = half_bits_to_float(lds_u16(base, blk + 208u));
  const float dl0 = d * static_cast<float>(static_cast<int8_t>(scw & 0xFFu)) * 64.f;
  const float dl1 = d * static_cast<float>(static_cast<int8_t>(scw >> 8)) * 64.f;
  const int shl = 4 * (u >> 1), shh = 2 * u;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ql[i] = (ql[i] >> shl) & 0x0F0F0F0Fu;  // this group's nibble in the low half of each byte
    qh[i] = (qh[i] >> shh) & 0x03030303u;  // this group's 2 high bits in bits 0..1 of each byte
  }
  uint32_t v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    // byte b of the words -> q6 at bits 17..22 of v
    v[4 * i + 0] = ((ql[i] << 17) & 0x001E0000u) | ((qh[i] << 21) & 0x00600000u) | kOne;
    v[4 * i + 1] = ((ql[i] << 9) & 0x001E0000u) | ((qh[i] << 13) & 0x00600000u) | kOne;
    v[4 * i + 2] = ((ql[i] << 1) & 0x001E0000u) | ((qh[i] << 5) & 0x00600000u) | kOne;
    v[4 * i + 3] = ((ql[i] >> 7) & 0x001E0000u) | ((qh[i] >> 3) & 0x00600000u) | kOne;
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float2 a0 = make_float2(-xs[t].s0, 0.f), a1 = make_float2(-xs[t].s1, 0.f);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      a0 = fma2(f2bits(v[j], v[j + 1]), xs[t].v[j >> 1], a0);
      a1 = fma2(f2bits(v[16 + j], v[17 + j]), xs[t].v[8 + (j >> 1)], a1);
    }
    // a = 2^-6 sum q6 x ; sum (q6-32) x = 64 a - 32 sum x
    out[t] += dl0 * ((a0.x + a0.y) - 0.5f * xs[t].s0) + dl1 * ((a1.x + a1.y) - 0.5f * xs[t].s1);
  }
}

template <int QT, int NT>
__device__ __forceinline__ void seg_dot(const uint32_t* base, uint32_t row, int seg, const XSeg* xs, float* out) {
  if (QT == kQ4_K) seg_dot_q4k<NT>(base, row, seg, xs, out);
  else if (QT == kQ4_0) seg_dot_q40<NT>(base, row, seg, xs, out);
  else if (QT == kQ8_0) seg_dot_q80<NT>(base, row, seg, xs, out);
  else seg_dot_q6k<NT>(base, row, seg, xs, out);
}

// ---- the kernel -------------------------------------------------------------
// SPT_C > 0: every thread owns exactly SPT_C segments and caches their
// activations for all M tokens in registers. SPT_C == 0: segments are visited
// in a runtime loop and activations are re-read (L1-resident) per tile/token.
template <int QT, int M, int SPT_C>
__global__ void __launch_bounds__(512) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, T = blockDim.x, nwarps = T >> 5, lane = tid & 31, warp = tid >> 5;
  const uint32_t* stage_words = reinterpret_cast<const uint32_t*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.stages * a.stage_bytes + 16);
  float* red = reinterpret_cast<float*>(full + a.stages);

  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();

  auto issue = [&](int64_t tile, int s) {
    const int64_t r0 = tile * a.rows;
    const int64_t nr = (a.n - r0) < a.rows ? (a.n - r0) : a.rows;
    const uint32_t bytes = static_cast<uint32_t>(nr * a.row_bytes);
    mbar_arrive_expect_tx(&full[s], bytes);
    bulk_g2s(smem + s * a.stage_bytes, a.q + r0 * a.row_bytes, bytes, &full[s]);
  };
  int64_t issued = 0;  // tiles issued by thread 0 (prologue + refills)
  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      const int64_t tile = blockIdx.x + static_cast<int64_t>(s) * gridDim.x;
      if (tile < a.ntiles) { issue(tile, s); ++issued; }
    }
  }

  constexpr int NC = SPT_C > 0 ? SPT_C : 1;
  constexpr int NTC = SPT_C > 0 ? M : 1;
  XSeg xc[NC][NTC];
  if (SPT_C > 0) {
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      const int seg = tid + j * T;
      if (seg < a.nseg) {
        int k0, k1;
        seg_k<QT>(seg, k0, k1);
#pragma unroll
        for (int t = 0; t < NTC; ++t) load_xseg(a.x, a.xtype, t * a.ldx, k0, k1, xc[j][t]);
      }
    }
  }
  const int spt = SPT_C > 0 ? SPT_C : (a.nseg + T - 1) / T;

  int it = 0;
  for (int64_t tile = blockIdx.x; tile < a.ntiles; tile += gridDim.x, ++it) {
    const int s = it % a.stages;
    const uint32_t par = static_cast<uint32_t>((it / a.stages) & 1);
    const bool ok = mbar_wait(&full[s], par);
    if (!__syncthreads_and(ok)) break;  // a wait gave up: unwind together

    const int64_t r0 = tile * a.rows;
    const int nr = static_cast<int>((a.n - r0) < a.rows ? (a.n - r0) : a.rows);
    const uint32_t sbase = static_cast<uint32_t>(s) * a.stage_bytes;
    float part[kRows][M];
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int t = 0; t < M; ++t) part[r][t] = 0.f;

    if constexpr (SPT_C > 0) {
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        const int seg = tid + j * T;
        if (seg < a.nseg) {
#pragma unroll
          for (int r = 0; r < kRows; ++r)
            if (r < nr) seg_dot<QT, M>(stage_words, sbase + r * static_cast<uint32_t>(a.row_bytes), seg, xc[j], part[r]);
        }
      }
    } else {
      for (int j = 0; j < spt; ++j) {
        const int seg = tid + j * T;
        if (seg >= a.nseg) break;
        int k0, k1;
        seg_k<QT>(seg, k0, k1);
#pragma unroll
        for (int t = 0; t < M; ++t) {
          XSeg xt;
          load_xseg(a.x, a.xtype, t * a.ldx, k0, k1, xt);
#pragma unroll
          for (int r = 0; r < kRows; ++r) {
            if (r < nr) {
              float o = 0.f;
              seg_dot<QT, 1>(stage_words, sbase + r * static_cast<uint32_t>(a.row_bytes), seg, &xt, &o);
              part[r][t] += o;
            }
          }
        }
      }
    }
    __syncthreads();  // stage s fully consumed
    if (tid == 0) {
      const int64_t nt = tile + static_cast<int64_t>(a.stages) * gridDim.x;
      if (nt < a.ntiles) { issue(nt, s); ++issued; }
    }
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int t = 0; t < M; ++t) {
        float v = part[r][t];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
        if (lane == 0) red[warp * (kRows * M) + r * M + t] = v;
      }
    __syncthreads();
    if (tid < kRows * M) {
      const int r = tid / M, t = tid - r * M;
      if (r < nr) {
        float v = 0.f;
        for (int w = 0; w < nwarps; ++w) v += red[w * (kRows * M) + tid];
        store_y_rt(a.y, a.ytype, t * a.ldy + r0 + r, v);
      }
    }
  }
  // On an early exit, drain every copy this CTA still has in flight (bounded).
  if (tid == 0) {
    const int64_t consumed = it;
    for (int64_t i = consumed; i < issued; ++i) {
      const int s = static_cast<int>(i % a.stages);
      mbar_wait(&full[s], static_cast<uint32_t>((i / a.stages) & 1));
    }
  }
}

// ---- host launch --------------------------------------------------------------
static std::mutex g_attr_mu;
static std::set<std::pair<const void*, int>> g_attr_done;

static cudaError_t ensure_smem_attr(const void* fn, int dev, int bytes) {
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (g_attr_done.count({fn, dev})) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) g_attr_done.insert({fn, dev});
  return e;
}

struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
};
DevInfo device_info(int dev);  // capi.cu

template <int QT, int M, int SPT_C>
static cudaError_t launch_gemv_t(const GemvArgs& a0, int threads, cudaStream_t st) {
  GemvArgs a = a0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const DevInfo di = device_info(dev);
  const int nwarps = threads / 32;
  const int extra = 16 + 8 * 4 + 4 * nwarps * kRows * M + 64;
  const int budget = std::min(di.smem_optin, 200 * 1024);
  // rows per tile: as many as fit (up to kRows) with at least 2 stages in flight
  int rows = kRows;
  while (rows > 1 && 2 * ((rows * a.row_bytes + 15) / 16 * 16) + extra > budget) --rows;
  a.rows = rows;
  a.stage_bytes = static_cast<uint32_t>((rows * a.row_bytes + 15) / 16 * 16);
  a.ntiles = (a.n + rows - 1) / rows;
  if (static_cast<int64_t>(a.stage_bytes) + extra > budget) return cudaErrorInvalidConfiguration;
  int stages = static_cast<int>(std::min<int64_t>(4, std::max<int64_t>(1, (budget - extra) / a.stage_bytes)));
  a.stages = stages;
  const int smem = static_cast<int>(stages * a.stage_bytes + extra);
  auto fn = gemv_kernel<QT, M, SPT_C>;
  e = ensure_smem_attr(reinterpret_cast<const void*>(fn), dev, std::min(di.smem_optin, 227 * 1024));
  if (e != cudaSuccess) return e;
  // Resident CTAs per SM from the smem / thread budgets (registers are <= 64
  // per thread for every variant, so threads bound first).
  int per_sm = std::max(1, std::min(2048 / threads, (228 * 1024) / (smem + 1024)));
  per_sm = std::min(per_sm, 32);
  const int64_t grid = std::min<int64_t>(a.ntiles, static_cast<int64_t>(di.sms) * per_sm);
  fn<<<static_cast<unsigned>(grid), threads, smem, st>>>(a);
  return cudaGetLastError();
}

template <int QT>
static cudaError_t launch_gemv_q(const GemvArgs& a, int m, int threads, int spt, cudaStream_t st) {
  if (m == 1 && spt == 1) return launch_gemv_t<QT, 1, 1>(a, threads, st);
  if (m == 1 && spt == 2) return launch_gemv_t<QT, 1, 2>(a, threads, st);
  if (m == 2 && spt == 1) return launch_gemv_t<QT, 2, 1>(a, threads, st);
  switch (m) {
    case 1: return launch_gemv_t<QT, 1, 0>(a, threads, st);
    case 2: return launch_gemv_t<QT, 2, 0>(a, threads, st);
    case 3: return launch_gemv_t<QT, 3, 0>(a, threads, st);
    case 4: return launch_gemv_t<QT, 4, 0>(a, threads, st);
    case 5: return launch_gemv_t<QT, 5, 0>(a, threads, st);
    case 6: return launch_gemv_t<QT, 6, 0>(a, threads, st);
    case 7: return launch_gemv_t<QT, 7, 0>(a, threads, st);
    case 8: return launch_gemv_t<QT, 8, 0>(a, threads, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t gemv_device_error(int* v, int clear, cudaStream_t st) { return tu_device_error(v, clear, st); }
cudaError_t gemv_set_wait_limit(uint32_t polls) { return tu_set_wait_limit(polls); }

// Preconditions (checked by the C-ABI): q 16-byte aligned, row_bytes % 16 == 0,
// x 16-byte aligned with ldx*elem % 16 == 0, 1 <= m <= 8.
cudaError_t launch_gemv(const void* q, int qtype, int64_t n, int64_t k, const void* x, int xtype, int64_t m,
                        int64_t ldx, void* y, int ytype, int64_t ldy, int64_t row_bytes, cudaStream_t st) {
  GemvArgs a{};
  a.q = static_cast<const uint8_t*>(q);
  a.n = n;
  a.row_bytes = row_bytes;
  a.x = x;
  a.ldx = ldx;
  a.y = y;
  a.ldy = ldy;
  a.xtype = xtype;
  a.ytype = ytype;
  a.nseg = static_cast<int>(k / 32);
  a.ntiles = (n + kRows - 1) / kRows;
  a.stage_bytes = static_cast<uint32_t>((kRows * row_bytes + 15) / 16 * 16);
  const int threads = std::min(512, (a.nseg + 31) / 32 * 32);
  const int spt = (a.nseg + threads - 1) / threads;
  switch (qtype) {
    case kQ4_0: return launch_gemv_q<kQ4_0>(a, static_cast<int>(m), threads, spt, st);
    case kQ8_0: return launch_gemv_q<kQ8_0>(a, static_cast<int>(m), threads, spt, st);
    case kQ4_K: return launch_gemv_q<kQ4_K>(a, static_cast<int>(m), threads, spt, st);
    case kQ6_K: return launch_gemv_q<kQ6_K>(a, static_cast<int>(m), threads, spt, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ggufmm
