// gemv_mma.cu -- decode GEMV (M <= 8 tokens) on the tensor cores, straight
// from GGUF blocks, for all four formats.
//
//   y[m, n] = sum_k x[m, k] W[n, k]
//
// Why tensor cores for a GEMV: the cost of a quantized GEMV at HBM speed is
// the per-weight decode work, not the multiply. On mma.sync.m16n8k16 the
// decode of two 4-bit quants is ONE lop3 ((w >> s) & 0x000F000F | 0x64006400
// is the fp16 pair 1024+q0, 1024+q1, exact), the multiply is 1/8 of an
// instruction per weight, and the unused token columns of the n8 tile are
// free, so M = 1..8 cost the same.
//
// Exactness: GGUF scales vary per 32 (Q6_K: 16) weights along K, so every
// sub-block's MMAs go into a fresh fp32 accumulator that is folded into the
// running sum with the sub-block's scale:
//     y += dsc * acc - (bias * dsc + dmin * m) * sum(x over the sub-block)
// where acc = sum x * (bias + q). Weights enter the dot product as exact
// integers and scales in fp32, so the result is as accurate as the fp32
// dequantize-then-matmul (not an fp16-rounded weight).
//
// Pipeline (warp-specialised, no block-wide barrier in the steady state):
//   producer warp   streams "pieces" (16 weight rows x one K chunk of <= 4096
//                   weights) into a ring of shared-memory stages with 1-D bulk
//                   TMA copies (one per row, completion on the stage's `full`
//                   mbarrier); a stage is refilled once every compute warp has
//                   arrived on its `empty` mbarrier.
//   compute warps   (W of them) each take every W-th 256-weight unit of a piece
//                   and keep 16 x 8 partial sums in registers across the chunks
//                   of a row block; at the end of a row block they park their
//                   partials in one of two reduction buffers (`rfull`).
//   epilogue warp   sums the W partials of a row block and writes y, then
//                   releases the buffer (`rempty`).
// The activations are converted once per CTA into fp16 in shared memory,
// permuted within groups of 8 ([0,2,1,3,4,6,5,7]) so every B fragment is one
// 128-bit load, with per-16/32 sums for the scale fold. fp32 activations are
// split into fp16 hi + lo columns. Token columns beyond M read column 0 and
// their results are never stored, so no load is predicated.
// Every mbarrier wait is bounded (kWaitLimit polls), flags g_device_error and
// unwinds instead of hanging.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace ggufmm {

constexpr int kRowsPerBlock = 16;
constexpr int kUnitK = 256;         // weights per unit (one K-quant superblock, 8 Q4_0/Q8_0 blocks)
constexpr int kMaxChunkUnits = 16;  // <= 4096 weights per piece
constexpr int kRedBufs = 2;
constexpr int kXsCols = 8;          // columns of the x-sum tables

struct MmaArgs {
  const uint8_t* q;
  int64_t n;
  int k;
  int64_t row_bytes;
  const void* x;
  int xtype;
  int64_t ldx;
  int m;     // tokens
  int cols;  // B columns in use: m (bf16/f16 x) or 2m (fp32 x split into hi + lo fp16)
  void* y;
  int ytype;
  int64_t ldy;
  int unit_bytes;
  int chunk_units;
  int nchunks;
  int chunk_bytes;  // bytes of one full chunk of one row
  int row_pitch;    // smem bytes per row inside a stage
  int stage_bytes;
  int stages;
  int64_t nrowblocks;
  int x_pitch;      // smem bytes per column of permuted fp16 x
  uint32_t x_off, xs32_off, xs16_off, red_off, bar_off;
};

// ---- small PTX helpers ---------------------------------------------------------
__device__ __forceinline__ uint32_t lop_and_or(uint32_t a, uint32_t m, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(m), "r"(c));  // (a & m) | c
  return d;
}
__device__ __forceinline__ uint32_t lop_and_xor(uint32_t a, uint32_t m, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(d) : "r"(a), "r"(m), "r"(c));  // (a & m) ^ c
  return d;
}

__device__ __forceinline__ void mma16816(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1, const float* c) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}
__device__ __forceinline__ void mma16816_z(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  const float z[4] = {0.f, 0.f, 0.f, 0.f};
  mma16816(d, a0, a1, a2, a3, b0, b1, z);
}

// Load 4 bytes from a 2-byte aligned shared-memory byte offset.
__device__ __forceinline__ uint32_t lds32_a2(const uint8_t* smem, uint32_t off) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(smem + (off & ~3u));
  return __funnelshift_r(w[0], w[1], (off & 3u) * 8u);
}
__device__ __forceinline__ uint32_t lds16(const uint8_t* smem, uint32_t off) {
  return *reinterpret_cast<const uint16_t*>(smem + off);
}

// Running sum fold for one sub-block: tot += dsc * acc - coef * xs.
// tot/acc layout (mma C fragment): [0,1] = row g, tokens 2t,2t+1; [2,3] = row g+8.
__device__ __forceinline__ void fold(float* tot, const float* acc, float dsc_g, float coef_g, float dsc_g8,
                                     float coef_g8, float2 xs) {
  tot[0] = fmaf(dsc_g, acc[0], fmaf(-coef_g, xs.x, tot[0]));
  tot[1] = fmaf(dsc_g, acc[1], fmaf(-coef_g, xs.y, tot[1]));
  tot[2] = fmaf(dsc_g8, acc[2], fmaf(-coef_g8, xs.x, tot[2]));
  tot[3] = fmaf(dsc_g8, acc[3], fmaf(-coef_g8, xs.y, tot[3]));
}

// fp16 pairs (bias + q) of the 4-bit fields of w: lo nibbles of bytes (0,2) / (1,3),
// hi nibbles of bytes (0,2) / (1,3).
struct Nib4 {
  uint32_t l02, l13, h02, h13;
};
__device__ __forceinline__ Nib4 nibbles(uint32_t w, uint32_t m0f, uint32_t k6400) {
  Nib4 r;
  r.l02 = lop_and_or(w, m0f, k6400);
  r.l13 = lop_and_or(w >> 8, m0f, k6400);
  r.h02 = lop_and_or(w >> 4, m0f, k6400);
  r.h13 = lop_and_or(w >> 12, m0f, k6400);
  return r;
}

// ---- per-format unit processing --------------------------------------------------
// A "unit" is 256 consecutive weights of a row: one Q4_K / Q6_K superblock or 8
// Q4_0 / Q8_0 blocks; sub-block j of the unit (32 weights, 16 for Q6_K) has the
// activations x[32j .. 32j+31] of the unit.
struct UnitCtx {
  const uint8_t* smem;
  uint32_t rg, rg8;   // smem byte offsets of the unit in rows g and g+8
  uint32_t xo;        // smem byte offset of this lane's x column at the unit's first k
  const float* xs32;  // x sums per 32 weights from the unit's first sub-block: [j][kXsCols]
  const float* xs16;  // ... per 16 weights (Q6_K only)
  int t, lane;
};

__device__ __forceinline__ uint4 ldx128(const UnitCtx& c, uint32_t kofs) {
  return *reinterpret_cast<const uint4*>(c.smem + c.xo + 2u * kofs);
}
__device__ __forceinline__ uint2 ldx64(const UnitCtx& c, uint32_t kofs) {
  return *reinterpret_cast<const uint2*>(c.smem + c.xo + 2u * kofs);
}
__device__ __forceinline__ float2 xs32(const UnitCtx& c, int j) {
  return *reinterpret_cast<const float2*>(c.xs32 + j * kXsCols + 2 * c.t);
}
__device__ __forceinline__ float2 xs16(const UnitCtx& c, int j) {
  return *reinterpret_cast<const float2*>(c.xs16 + j * kXsCols + 2 * c.t);
}

// Q4_K: 8 sub-blocks of 32; chunk ch (0..3) = 32 qs bytes at 16+32ch, low nibbles ->
// sub-block 2ch, high -> 2ch+1. Thread t takes bytes 8t..8t+7 of each chunk and
// decodes the scales of sub-blocks 2t, 2t+1, shared with the quad by shuffles.
__device__ __forceinline__ void unit_q4k(const UnitCtx& c, float* tot, uint32_t m0f, uint32_t k6400) {
  const uint4 hg = *reinterpret_cast<const uint4*>(c.smem + c.rg);
  const uint4 hg8 = *reinterpret_cast<const uint4*>(c.smem + c.rg8);
  float sv[8];  // [row][which][dsc, coef]
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint4 h = r == 0 ? hg : hg8;
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    // 6-bit scales/mins (gguf quants.py:479-501), four sub-blocks per word:
    //   0..3: sc = s[j] & 63,  m = s[j+4] & 63
    //   4..7: sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4,  m = (s[j+4] >> 4) | (s[j] >> 6) << 4
    const uint32_t scw = c.t < 2 ? (h.y & 0x3F3F3F3Fu) : ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u));
    const uint32_t mw = c.t < 2 ? (h.z & 0x3F3F3F3Fu) : (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u));
    const uint32_t sh = 16u * (c.t & 1);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float ds = d * static_cast<float>((scw >> (sh + 8 * i)) & 0xFFu);
      sv[4 * r + 2 * i] = ds;
      sv[4 * r + 2 * i + 1] = fmaf(1024.f, ds, dmin * static_cast<float>((mw >> (sh + 8 * i)) & 0xFFu));
    }
  }
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    const int src = (c.lane & ~3) | ch;
    float s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = __shfl_sync(0xFFFFFFFFu, sv[i], src);
    const uint2 wg = *reinterpret_cast<const uint2*>(c.smem + c.rg + 16u + 32u * ch + 8u * c.t);
    const uint2 wg8 = *reinterpret_cast<const uint2*>(c.smem + c.rg8 + 16u + 32u * ch + 8u * c.t);
    const uint4 xl = ldx128(c, 64u * ch + 8u * c.t);
    const uint4 xh = ldx128(c, 64u * ch + 32u + 8u * c.t);
    const Nib4 a0 = nibbles(wg.x, m0f, k6400), a1 = nibbles(wg8.x, m0f, k6400);
    const Nib4 b0 = nibbles(wg.y, m0f, k6400), b1 = nibbles(wg8.y, m0f, k6400);
    float accl[4], acch[4];
    mma16816_z(accl, a0.l02, a1.l02, a0.l13, a1.l13, xl.x, xl.y);
    mma16816(accl, b0.l02, b1.l02, b0.l13, b1.l13, xl.z, xl.w, accl);
    mma16816_z(acch, a0.h02, a1.h02, a0.h13, a1.h13, xh.x, xh.y);
    mma16816(acch, b0.h02, b1.h02, b0.h13, b1.h13, xh.z, xh.w, acch);
    fold(tot, accl, s[0], s[1], s[4], s[5], xs32(c, 2 * ch));
    fold(tot + 4, acch, s[2], s[3], s[6], s[7], xs32(c, 2 * ch + 1));
  }
}

// Q4_0: 8 blocks of 18 bytes (fp16 d + 16 nibble bytes; byte i: low nibble ->
// x[i], high -> x[16+i]); value d*(q-8). Thread t takes bytes 4t..4t+3.
__device__ __forceinline__ void unit_q40(const UnitCtx& c, float* tot, uint32_t m0f, uint32_t k6400) {
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const uint32_t og = c.rg + 18u * b, og8 = c.rg8 + 18u * b;
    const float dg = half_bits_to_float(lds16(c.smem, og)), dg8 = half_bits_to_float(lds16(c.smem, og8));
    const uint32_t wg = lds32_a2(c.smem, og + 2u + 4u * c.t), wg8 = lds32_a2(c.smem, og8 + 2u + 4u * c.t);
    const uint2 xl = ldx64(c, 32u * b + 4u * c.t);
    const uint2 xh = ldx64(c, 32u * b + 16u + 4u * c.t);
    const Nib4 a = nibbles(wg, m0f, k6400), a8 = nibbles(wg8, m0f, k6400);
    float acc[4];
    mma16816_z(acc, a.l02, a8.l02, a.l13, a8.l13, xl.x, xl.y);
    mma16816(acc, a.h02, a8.h02, a.h13, a8.h13, xh.x, xh.y, acc);
    fold(tot + 4 * (b & 1), acc, dg, 1032.f * dg, dg8, 1032.f * dg8, xs32(c, b));
  }
}

// Q8_0: 8 blocks of 34 bytes (fp16 d + 32 int8); q+128 as fp16 (1152 + q).
// Thread t takes bytes 4t..4t+3 (k16 step 0) and 16+4t.. (step 1) of each block.
__device__ __forceinline__ void unit_q80(const UnitCtx& c, float* tot) {
  const uint32_t mff = 0x00FF00FFu, kx = 0x64806480u;  // (w & 0x00FF00FF) ^ 0x64806480 = 0x64.. | (byte ^ 0x80)
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const uint32_t og = c.rg + 34u * b, og8 = c.rg8 + 34u * b;
    const float dg = half_bits_to_float(lds16(c.smem, og)), dg8 = half_bits_to_float(lds16(c.smem, og8));
    const uint32_t w0 = lds32_a2(c.smem, og + 2u + 4u * c.t), w1 = lds32_a2(c.smem, og + 18u + 4u * c.t);
    const uint32_t v0 = lds32_a2(c.smem, og8 + 2u + 4u * c.t), v1 = lds32_a2(c.smem, og8 + 18u + 4u * c.t);
    const uint2 x0 = ldx64(c, 32u * b + 4u * c.t);
    const uint2 x1 = ldx64(c, 32u * b + 16u + 4u * c.t);
    float acc[4];
    mma16816_z(acc, lop_and_xor(w0, mff, kx), lop_and_xor(v0, mff, kx), lop_and_xor(w0 >> 8, mff, kx),
               lop_and_xor(v0 >> 8, mff, kx), x0.x, x0.y);
    mma16816(acc, lop_and_xor(w1, mff, kx), lop_and_xor(v1, mff, kx), lop_and_xor(w1 >> 8, mff, kx),
             lop_and_xor(v1 >> 8, mff, kx), x1.x, x1.y, acc);
    fold(tot + 4 * (b & 1), acc, dg, 1152.f * dg, dg8, 1152.f * dg8, xs32(c, b));
  }
}

// Q6_K: element e = 128h + 32u + cc (h = 0..1, u = 0..3, cc = 0..31):
// q6 = (ql[64h + 32(u&1) + cc] >> 4(u>>1)) & 15 | ((qh[128 + 32h + cc] >> 2u) & 3) << 4,
// value = (d * sc[e/16]) * (q6 - 32). One k16 step = one 16-weight scale group;
// thread t takes elements cc = 16s + 4t .. +3.
__device__ __forceinline__ void unit_q6k(const UnitCtx& c, float* tot, uint32_t k6400) {
  const float dg = half_bits_to_float(lds16(c.smem, c.rg + 208u));
  const float dg8 = half_bits_to_float(lds16(c.smem, c.rg8 + 208u));
  const uint32_t m0f = 0x000F000Fu, m30 = 0x00300030u;
#pragma unroll
  for (int grp = 0; grp < 8; ++grp) {  // 32-element group = 128h + 32u
    const int h = grp >> 2, u = grp & 3;
    const uint32_t qlo = 64u * h + 32u * (u & 1), qho = 128u + 32u * h;
    const int shl = 4 * (u >> 1), shh = 2 * u;
    const uint32_t scg = lds16(c.smem, c.rg + 192u + 2u * grp), scg8 = lds16(c.smem, c.rg8 + 192u + 2u * grp);
#pragma unroll
    for (int s = 0; s < 2; ++s) {  // 16-element scale group 2*grp + s
      const uint32_t cc = 16u * s + 4u * c.t;
      const uint32_t lg = lds32_a2(c.smem, c.rg + qlo + cc) >> shl, lg8 = lds32_a2(c.smem, c.rg8 + qlo + cc) >> shl;
      const uint32_t hg = lds32_a2(c.smem, c.rg + qho + cc) >> shh, hg8 = lds32_a2(c.smem, c.rg8 + qho + cc) >> shh;
      // bytes (0,2) and (1,3): (nibble | hi2 << 4) | 0x6400 = fp16 1024 + q6
      const uint32_t a0 = lop_and_or(lg, m0f, lop_and_or(hg << 4, m30, k6400));
      const uint32_t a2 = lop_and_or(lg >> 8, m0f, lop_and_or(hg >> 4, m30, k6400));
      const uint32_t a1 = lop_and_or(lg8, m0f, lop_and_or(hg8 << 4, m30, k6400));
      const uint32_t a3 = lop_and_or(lg8 >> 8, m0f, lop_and_or(hg8 >> 4, m30, k6400));
      const uint2 xb = ldx64(c, 32u * grp + cc);
      float acc[4];
      mma16816_z(acc, a0, a1, a2, a3, xb.x, xb.y);
      const float dl = dg * static_cast<float>(static_cast<int8_t>(scg >> (8 * s)));
      const float dl8 = dg8 * static_cast<float>(static_cast<int8_t>(scg8 >> (8 * s)));
      fold(tot + 4 * s, acc, dl, 1056.f * dl, dl8, 1056.f * dl8, xs16(c, 2 * grp + s));  // bias 1024 + 32
    }
  }
}

template <int QT>
__device__ __forceinline__ void process_unit(const UnitCtx& c, float* tot) {
  const uint32_t m0f = 0x000F000Fu, k6400 = 0x64006400u;
  if (QT == kQ4_K) unit_q4k(c, tot, m0f, k6400);
  else if (QT == kQ4_0) unit_q40(c, tot, m0f, k6400);
  else if (QT == kQ8_0) unit_q80(c, tot);
  else unit_q6k(c, tot, k6400);
}

// ---- the kernel ---------------------------------------------------------------------
__device__ __forceinline__ uint32_t perm8(uint32_t e) { return (e & 4u) | ((e & 1u) << 1) | ((e >> 1) & 1u); }

// W compute warps + 1 producer warp + 1 epilogue warp.
template <int QT, int W>
__global__ void __launch_bounds__((W + 2) * 32, 1) gemv_mma_kernel(const MmaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  constexpr int kThreads = (W + 2) * 32;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.bar_off);
  uint64_t* empty = full + a.stages;
  uint64_t* rfull = empty + a.stages;
  uint64_t* rempty = rfull + kRedBufs;
  float* xs32t = reinterpret_cast<float*>(smem + a.xs32_off);
  float* xs16t = reinterpret_cast<float*>(smem + a.xs16_off);
  float* red = reinterpret_cast<float*>(smem + a.red_off);  // [kRedBufs][W][16 rows][8 cols]
  const int64_t my_blocks = a.nrowblocks > blockIdx.x ? (a.nrowblocks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t total_pieces = my_blocks * a.nchunks;
  const int total_units = a.k / kUnitK;

  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    for (int b = 0; b < kRedBufs; ++b) {
      mbar_init(&rfull[b], W);
      mbar_init(&rempty[b], 1);
    }
    fence_mbar_init();
  }

  // activations -> permuted fp16 [cols][k]; sums per 16 / 32 weights, [k/16][8] / [k/32][8]
  {
    const int groups = a.k / 8;  // 8 consecutive k per task
    const int nparts = a.xtype == GGUFMM_F32 ? 2 : 1;
    for (int task = tid; task < a.m * groups; task += kThreads) {
      const int tok = task / groups, k0 = (task - tok * groups) * 8;
      float v[8];
      if (a.xtype == GGUFMM_F32) {
        const float* xp = static_cast<const float*>(a.x) + tok * a.ldx + k0;
        const float4 p0 = *reinterpret_cast<const float4*>(xp), p1 = *reinterpret_cast<const float4*>(xp + 4);
        v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w; v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
      } else {
        const uint4 p = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.x) + tok * a.ldx + k0);
        const uint32_t w[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (a.xtype == GGUFMM_BF16) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
          } else {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
          }
        }
      }
      for (int part = 0; part < nparts; ++part) {
        __half hv[8];
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const __half hi = __float2half_rn(v[e]);
          const __half hh = part == 0 ? hi : __float2half_rn(v[e] - __half2float(hi));
          hv[perm8(e)] = hh;
          s += __half2float(hh);
        }
        const int col = tok + part * a.m;
        *reinterpret_cast<uint4*>(smem + a.x_off + col * a.x_pitch + 2 * k0) = *reinterpret_cast<uint4*>(hv);
        s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);  // 16 weights = two adjacent tasks
        if (QT == kQ6_K && (task & 1) == 0) xs16t[(k0 / 16) * kXsCols + col] = s;
        s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);  // 32 weights = four adjacent tasks
        if ((task & 3) == 0) xs32t[(k0 / 32) * kXsCols + col] = s;
      }
    }
  }
  __syncthreads();

  if (warp == W) {
    // ---------------- producer ----------------
    if (lane == 0) {
      for (int64_t p = 0; p < total_pieces; ++p) {
        const int s = static_cast<int>(p % a.stages);
        if (p >= a.stages && !mbar_wait(&empty[s], static_cast<uint32_t>(((p / a.stages) - 1) & 1))) break;
        const int64_t rb = blockIdx.x + (p / a.nchunks) * gridDim.x;
        const int ch = static_cast<int>(p % a.nchunks);
        const int64_t r0 = rb * kRowsPerBlock;
        const int nr = static_cast<int>((a.n - r0) < kRowsPerBlock ? (a.n - r0) : kRowsPerBlock);
        const int units = min(a.chunk_units, total_units - ch * a.chunk_units);
        const uint32_t bytes = static_cast<uint32_t>(units * a.unit_bytes);
        mbar_arrive_expect_tx(&full[s], bytes * nr);
        uint8_t* dst = smem + s * a.stage_bytes;
        const uint8_t* src = a.q + r0 * a.row_bytes + static_cast<int64_t>(ch) * a.chunk_bytes;
        for (int r = 0; r < nr; ++r) bulk_g2s(dst + r * a.row_pitch, src + r * a.row_bytes, bytes, &full[s]);
      }
    }
  } else if (warp == W + 1) {
    // ---------------- epilogue ----------------
    for (int64_t blk = 0; blk < my_blocks; ++blk) {
      const int b = static_cast<int>(blk & 1);
      if (!mbar_wait(&rfull[b], static_cast<uint32_t>((blk >> 1) & 1))) break;
      const int64_t rb = blockIdx.x + blk * gridDim.x;
      const float* rbuf = red + b * (W * kRowsPerBlock * 8);
      for (int i = lane; i < kRowsPerBlock * a.m; i += 32) {
        const int row = i / a.m, tok = i - row * a.m;
        const int64_t n_idx = rb * kRowsPerBlock + row;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) {
          v += rbuf[(w * kRowsPerBlock + row) * 8 + tok];
          if (a.cols > a.m) v += rbuf[(w * kRowsPerBlock + row) * 8 + tok + a.m];
        }
        if (n_idx < a.n) store_y_rt(a.y, a.ytype, tok * a.ldy + n_idx, v);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rempty[b]);
    }
  } else {
    // ---------------- compute ----------------
    const uint32_t xcol = a.x_off + (g < a.cols ? g : 0) * a.x_pitch;
    float tot[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // two independent fold chains
    int64_t p = 0;
    bool ok = true;
    for (int64_t blk = 0; blk < my_blocks && ok; ++blk) {
      for (int ch = 0; ch < a.nchunks; ++ch, ++p) {
        const int s = static_cast<int>(p % a.stages);
        if (!mbar_wait(&full[s], static_cast<uint32_t>((p / a.stages) & 1))) {
          ok = false;
          break;
        }
        const int units = min(a.chunk_units, total_units - ch * a.chunk_units);
        const uint32_t sbase = static_cast<uint32_t>(s * a.stage_bytes) + g * a.row_pitch;
        for (int u = warp; u < units; u += W) {
          const int ku = (ch * a.chunk_units + u) * kUnitK;
          UnitCtx c;
          c.smem = smem;
          c.rg = sbase + u * a.unit_bytes;
          c.rg8 = c.rg + 8 * a.row_pitch;
          c.xo = xcol + 2u * ku;
          c.xs32 = xs32t + (ku / 32) * kXsCols;
          c.xs16 = xs16t + (ku / 16) * kXsCols;
          c.t = t;
          c.lane = lane;
          process_unit<QT>(c, tot);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with stage s
      }
      if (!ok) break;
      // row block complete: park the partial 16 x 8 tile for the epilogue
      const int b = static_cast<int>(blk & 1);
      if (blk >= kRedBufs && !mbar_wait(&rempty[b], static_cast<uint32_t>(((blk >> 1) - 1) & 1))) break;
      float* rw = red + b * (W * kRowsPerBlock * 8) + warp * (kRowsPerBlock * 8);
      *reinterpret_cast<float2*>(rw + g * 8 + 2 * t) = make_float2(tot[0] + tot[4], tot[1] + tot[5]);
      *reinterpret_cast<float2*>(rw + (g + 8) * 8 + 2 * t) = make_float2(tot[2] + tot[6], tot[3] + tot[7]);
#pragma unroll
      for (int i = 0; i < 8; ++i) tot[i] = 0.f;
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfull[b]);
    }
  }
  __syncthreads();
  // A bounded wait may have given up (g_device_error is set): make sure no copy
  // of this CTA is still in flight before it exits.
  if (warp == W && lane == 0) {
    for (int64_t q = total_pieces - a.stages; q < total_pieces; ++q)
      if (q >= 0) mbar_wait(&full[q % a.stages], static_cast<uint32_t>((q / a.stages) & 1));
  }
}

// ---- host side ------------------------------------------------------------------------
struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
};
DevInfo device_info(int dev);  // capi.cu

static std::mutex g_mma_attr_mu;
static std::set<std::pair<const void*, int>> g_mma_attr_done;

static int unit_bytes_of(int qt) {
  switch (qt) {
    case kQ4_K: return 144;
    case kQ6_K: return 210;
    case kQ4_0: return 8 * 18;
    case kQ8_0: return 8 * 34;
    default: return 0;
  }
}

// Compute warps per CTA (8 by default; GGUFMM_GEMV_WARPS=4|16 for tuning).
static int compute_warps() {
  static const int w = [] {
    const char* e = std::getenv("GGUFMM_GEMV_WARPS");
    const int v = e ? std::atoi(e) : 8;
    return v == 16 ? 16 : (v == 4 ? 4 : 8);
  }();
  return w;
}

// Whether the tensor-core GEMV handles this problem; fills the launch plan.
static bool plan_mma(int qt, int64_t n, int64_t k, int m, int xtype, int smem_budget, int W, MmaArgs& a) {
  a.unit_bytes = unit_bytes_of(qt);
  if (!a.unit_bytes || k % kUnitK || m < 1 || m > 8) return false;
  a.cols = xtype == GGUFMM_F32 ? 2 * m : m;
  if (a.cols > 8) return false;
  const int units = static_cast<int>(k / kUnitK);
  // Q6_K superblocks are 210 bytes: copies stay 16-byte multiples only for 8-unit chunks
  const int align_units = qt == kQ6_K ? 8 : 1;
  if (units % align_units) return false;
  a.chunk_units = std::min(units, kMaxChunkUnits);
  a.chunk_units -= a.chunk_units % align_units;
  a.nchunks = (units + a.chunk_units - 1) / a.chunk_units;
  a.chunk_bytes = a.chunk_units * a.unit_bytes;
  if (a.chunk_bytes % 16) return false;
  a.row_pitch = (a.chunk_bytes + 127) / 128 * 128 + 32;  // pitch = 32 mod 128: conflict-free 8-byte row reads
  a.stage_bytes = kRowsPerBlock * a.row_pitch;
  a.x_pitch = static_cast<int>(2 * k + 64);
  const int x_bytes = a.cols * a.x_pitch;
  const int xs32_bytes = static_cast<int>(k / 32) * kXsCols * 4;
  const int xs16_bytes = qt == kQ6_K ? static_cast<int>(k / 16) * kXsCols * 4 : 0;
  const int red_bytes = kRedBufs * W * kRowsPerBlock * 8 * 4;
  const int fixed = x_bytes + xs32_bytes + xs16_bytes + red_bytes + 16 * 8 + 64;
  const int stages = std::min(6, (smem_budget - fixed) / a.stage_bytes);
  if (stages < 2) return false;
  a.stages = stages;
  a.x_off = static_cast<uint32_t>(stages * a.stage_bytes);
  a.xs32_off = a.x_off + x_bytes;
  a.xs16_off = a.xs32_off + xs32_bytes;
  a.red_off = a.xs16_off + xs16_bytes;
  a.bar_off = (a.red_off + red_bytes + 7) / 8 * 8;
  a.nrowblocks = (n + kRowsPerBlock - 1) / kRowsPerBlock;
  return true;
}

bool gemv_mma_supported(int qtype, int64_t n, int64_t k, int m, int xtype) {
  MmaArgs a{};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const DevInfo di = device_info(dev);
  return plan_mma(qtype, n, k, m, xtype, std::min(di.smem_optin, 227 * 1024), compute_warps(), a);
}

template <int QT, int W>
static cudaError_t launch_mma_t(MmaArgs& a, int dev, const DevInfo& di, cudaStream_t st) {
  auto fn = gemv_mma_kernel<QT, W>;
  const int smem = static_cast<int>(a.bar_off + 8 * (2 * a.stages + 2 * kRedBufs));
  {
    std::lock_guard<std::mutex> lk(g_mma_attr_mu);
    if (!g_mma_attr_done.count({reinterpret_cast<const void*>(fn), dev})) {
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           std::min(di.smem_optin, 227 * 1024));
      if (e != cudaSuccess) return e;
      g_mma_attr_done.insert({reinterpret_cast<const void*>(fn), dev});
    }
  }
  const int64_t grid = std::min<int64_t>(a.nrowblocks, di.sms);
  fn<<<static_cast<unsigned>(grid), (W + 2) * 32, smem, st>>>(a);
  return cudaGetLastError();
}

template <int QT>
static cudaError_t launch_mma_q(MmaArgs& a, int W, int dev, const DevInfo& di, cudaStream_t st) {
  if (W == 16) return launch_mma_t<QT, 16>(a, dev, di, st);
  if (W == 4) return launch_mma_t<QT, 4>(a, dev, di, st);
  return launch_mma_t<QT, 8>(a, dev, di, st);
}

cudaError_t launch_gemv_mma(const void* q, int qtype, int64_t n, int64_t k, const void* x, int xtype, int64_t m,
                            int64_t ldx, void* y, int ytype, int64_t ldy, int64_t row_bytes, cudaStream_t st) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const DevInfo di = device_info(dev);
  const int W = compute_warps();
  MmaArgs a{};
  if (!plan_mma(qtype, n, k, static_cast<int>(m), xtype, std::min(di.smem_optin, 227 * 1024), W, a))
    return cudaErrorInvalidValue;
  a.q = static_cast<const uint8_t*>(q);
  a.n = n;
  a.k = static_cast<int>(k);
  a.row_bytes = row_bytes;
  a.x = x;
  a.xtype = xtype;
  a.ldx = ldx;
  a.m = static_cast<int>(m);
  a.y = y;
  a.ytype = ytype;
  a.ldy = ldy;
  switch (qtype) {
    case kQ4_K: return launch_mma_q<kQ4_K>(a, W, dev, di, st);
    case kQ4_0: return launch_mma_q<kQ4_0>(a, W, dev, di, st);
    case kQ8_0: return launch_mma_q<kQ8_0>(a, W, dev, di, st);
    case kQ6_K: return launch_mma_q<kQ6_K>(a, W, dev, di, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t gemv_mma_device_error(int* v, int clear, cudaStream_t st) { return tu_device_error(v, clear, st); }

}  // namespace ggufmm
