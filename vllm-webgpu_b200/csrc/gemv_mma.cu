// gemv_mma.cu -- decode GEMV (M <= 8 tokens) on the tensor cores, straight
// from GGUF blocks, for all four formats.
//
//   y[m, n] = sum_k x[m, k] W[n, k]
//
// Why tensor cores for a GEMV: the cost of a quantized GEMV at HBM speed is
// the per-weight decode work, not the multiply. On mma.sync.m16n8k16 a pair of
// 4-bit quants becomes an fp16 operand with ONE lop3: (w >> s) & 0x000F000F is
// the pair q0 * 2^-24, q2 * 2^-24 as fp16 subnormals, exact (Q4_K high nibbles
// are used unshifted, & 0x00F000F0 = 16 q * 2^-24). The multiply is 1/8 of an
// instruction per weight and the unused token columns of the n8 tile are free,
// so M = 1..8 cost the same.
//
// Exactness: GGUF scales vary per 32 (Q6_K: 16) weights along K, so every
// scale group's MMAs go into a fresh fp32 accumulator that is folded into the
// running sum with the group's scale (2^24 folded in): tot += dsc * acc. The
// group's offset / min part, coef_j * sum(x over group j) (Q4_K: dmin m_j,
// Q4_0: 8 d, Q8_0: 128 d, Q6_K: 32 d sc_j), is a small matrix product of its
// own and also runs on the tensor core (bf16 hi/lo splits, accumulated over the
// row block). Weights enter as exact integers and scales in fp32, so the result
// is as accurate as the fp32 dequantize-then-matmul (not an fp16-rounded
// weight).
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

// One weight of a grouped launch: several weights with the same K that read the
// same activations (fused q/k/v, gate/up) share one launch; their row blocks are
// numbered consecutively, segment i owning row blocks [rb0, next rb0).
constexpr int kMaxSegs = 4;
struct MmaSeg {
  const uint8_t* q;
  void* y;
  int64_t n;
  int64_t ldy;
  int64_t rb0;
};

struct MmaArgs {
  MmaSeg seg[kMaxSegs];
  int nseg;
  int k;
  int64_t row_bytes;
  const void* x;
  int xtype;
  int64_t ldx;
  int m;     // tokens
  int cols;  // B columns in use: m (bf16/f16 x) or 2m (fp32 x split into hi + lo fp16)
  int ytype;
  int unit_bytes;
  int chunk_units;
  int nchunks;
  int chunk_bytes;  // bytes of one full chunk of one row
  int row_pitch;    // smem bytes per row inside a stage
  int stage_bytes;
  int stages;
  int64_t nrowblocks;
  int x_pitch;      // smem bytes per column of permuted fp16 x
  int lead;         // rows not 16-byte multiples (Q6_K, K/256 not a multiple of 8): each row's
                    // copy starts at its 16-byte aligned-down address, the row (row_start & 15)
                    // bytes into its smem slot
  uint32_t x_off, xsb_off, xsb_lo, red_off, bar_off;  // xsb: bf16 x-sum slots, lo part at +xsb_lo
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

// fp16 pairs of the 4-bit fields of w (or-ed with k, 0 here: fp16 subnormals q * 2^-24):
// lo nibbles of bytes (0,2) / (1,3), hi nibbles of bytes (0,2) / (1,3).
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
// Q4_0 / Q8_0 blocks. Its scale groups (8 sub-blocks of 32, or 16 groups of 16
// for Q6_K) each get a fresh MMA accumulator folded with tot += dsc * acc. The
// offset / min part of every group, coef_j * sum(x over group j), is itself a small
// matrix product: coef [16 rows x 16 group slots] times x-sums [16 slots x 8
// columns]. It runs on the tensor core too (bf16 hi/lo splits of both operands,
// three MMAs, accurate to ~2^-16), accumulating into `cm` over the whole row
// block; the row block's result is tot - cm.
struct UnitCtx {
  const uint8_t* smem;
  uint32_t rg, rg8;  // smem byte offsets of the unit in rows g and g+8
  uint32_t xo;       // smem byte offset of this lane's x column at the unit's first k
  uint32_t xsh;      // smem byte offset of this lane's (unit, column, t) x-sum slots, bf16 hi part
  uint32_t xsl_add;  // + this = lo part
  int t, lane;
};

__device__ __forceinline__ uint4 ldx128(const UnitCtx& c, uint32_t kofs) {
  return *reinterpret_cast<const uint4*>(c.smem + c.xo + 2u * kofs);
}
__device__ __forceinline__ uint2 ldx64(const UnitCtx& c, uint32_t kofs) {
  return *reinterpret_cast<const uint2*>(c.smem + c.xo + 2u * kofs);
}

__device__ __forceinline__ void mma_bf16(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bf16x2 hi / lo split of (a, b): a = hi.x + lo.x to ~2^-16 relative.
__device__ __forceinline__ void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const float2 hf = __bfloat1622float2(h);
  const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// cm += coef . xsums for the unit. coef pairs: (row g, slots 2t,2t+1), (row g+8, ..),
// (row g, slots 2t+8,2t+9), (row g+8, ..); zero where a format has 8 groups.
__device__ __forceinline__ void coef_mma(const UnitCtx& c, float* cm, float2 cg, float2 cg8, float2 cg_hi,
                                         float2 cg8_hi) {
  uint32_t a0h, a0l, a1h, a1l, a2h, a2l, a3h, a3l;
  split2(cg.x, cg.y, a0h, a0l);
  split2(cg8.x, cg8.y, a1h, a1l);
  split2(cg_hi.x, cg_hi.y, a2h, a2l);
  split2(cg8_hi.x, cg8_hi.y, a3h, a3l);
  const uint2 bh = *reinterpret_cast<const uint2*>(c.smem + c.xsh);
  const uint2 bl = *reinterpret_cast<const uint2*>(c.smem + c.xsh + c.xsl_add);
  mma_bf16(cm, a0h, a1h, a2h, a3h, bh.x, bh.y);
  mma_bf16(cm, a0h, a1h, a2h, a3h, bl.x, bl.y);
  mma_bf16(cm, a0l, a1l, a2l, a3l, bh.x, bh.y);
}

// tot += d * acc (rows g -> [0,1], g+8 -> [2,3])
__device__ __forceinline__ void fold_d(float* tot, const float* acc, float d_g, float d_g8) {
  tot[0] = fmaf(d_g, acc[0], tot[0]);
  tot[1] = fmaf(d_g, acc[1], tot[1]);
  tot[2] = fmaf(d_g8, acc[2], tot[2]);
  tot[3] = fmaf(d_g8, acc[3], tot[3]);
}

// Q4_K: 8 sub-blocks of 32; chunk ch (0..3) = 32 qs bytes at 16+32ch, low nibbles ->
// sub-block 2ch, high -> 2ch+1. Thread t takes bytes 8t..8t+7 of each chunk. Low
// nibbles enter the MMA as q * 2^-24, high nibbles unshifted as 16 q * 2^-24. Thread t
// decodes the scales of sub-blocks 2t, 2t+1 and shares the dsc values with its quad.
__device__ __forceinline__ void unit_q4k(const UnitCtx& c, float* tot, float* cm) {
  const uint32_t m0f = 0x000F000Fu, mf0 = 0x00F000F0u, k6400 = 0u;  // quants as fp16 subnormals q*2^-24
  const uint4 hg = *reinterpret_cast<const uint4*>(c.smem + c.rg);
  const uint4 hg8 = *reinterpret_cast<const uint4*>(c.smem + c.rg8);
  float sv[4];    // [row][lo dsc, hi dsc/16]
  float2 cf[2];   // [row] (coef of sub-block 2t, coef of 2t+1)
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint4 h = r == 0 ? hg : hg8;
    const float d = half_bits_to_float(h.x), dmin = half_bits_to_float(h.x >> 16);
    // 6-bit scales/mins (gguf quants.py:479-501), four sub-blocks per word:
    //   0..3: sc = s[j] & 63,  m = s[j+4] & 63
    //   4..7: sc = (s[j+4] & 15) | (s[j-4] >> 6) << 4,  m = (s[j+4] >> 4) | (s[j] >> 6) << 4
    // (branch-free: lanes of a warp differ in t)
    const uint32_t hi_sel = 0u - static_cast<uint32_t>(c.t >> 1);  // all ones for t >= 2
    const uint32_t scw = ((h.y & 0x3F3F3F3Fu) & ~hi_sel) | (((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u)) & hi_sel);
    const uint32_t mw = ((h.z & 0x3F3F3F3Fu) & ~hi_sel) | ((((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u)) & hi_sel);
    const uint32_t sh = 16u * (c.t & 1);
    const float dlo = d * static_cast<float>((scw >> sh) & 0xFFu);
    const float dhi = d * static_cast<float>((scw >> (sh + 8)) & 0xFFu);
    // lows: acc = 2^-24 sum x q, highs (unshifted) acc = 2^-20 sum x q; min term dmin m xs
    sv[2 * r] = dlo * 16777216.f;
    sv[2 * r + 1] = dhi * 1048576.f;
    cf[r] = make_float2(dmin * static_cast<float>((mw >> sh) & 0xFFu), dmin * static_cast<float>((mw >> (sh + 8)) & 0xFFu));
  }
  coef_mma(c, cm, cf[0], cf[1], make_float2(0.f, 0.f), make_float2(0.f, 0.f));
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    const int src = (c.lane & ~3) | ch;
    float s[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) s[i] = __shfl_sync(0xFFFFFFFFu, sv[i], src);
    const uint2 wg = *reinterpret_cast<const uint2*>(c.smem + c.rg + 16u + 32u * ch + 8u * c.t);
    const uint2 wg8 = *reinterpret_cast<const uint2*>(c.smem + c.rg8 + 16u + 32u * ch + 8u * c.t);
    const uint4 xl = ldx128(c, 64u * ch + 8u * c.t);
    const uint4 xh = ldx128(c, 64u * ch + 32u + 8u * c.t);
    const uint32_t g0 = wg.x, g1 = wg.y, h0 = wg8.x, h1 = wg8.y;
    const uint32_t g0s = g0 >> 8, g1s = g1 >> 8, h0s = h0 >> 8, h1s = h1 >> 8;
    float accl[4], acch[4];
    mma16816_z(accl, lop_and_or(g0, m0f, k6400), lop_and_or(h0, m0f, k6400), lop_and_or(g0s, m0f, k6400),
               lop_and_or(h0s, m0f, k6400), xl.x, xl.y);
    mma16816(accl, lop_and_or(g1, m0f, k6400), lop_and_or(h1, m0f, k6400), lop_and_or(g1s, m0f, k6400),
             lop_and_or(h1s, m0f, k6400), xl.z, xl.w, accl);
    mma16816_z(acch, lop_and_or(g0, mf0, k6400), lop_and_or(h0, mf0, k6400), lop_and_or(g0s, mf0, k6400),
               lop_and_or(h0s, mf0, k6400), xh.x, xh.y);
    mma16816(acch, lop_and_or(g1, mf0, k6400), lop_and_or(h1, mf0, k6400), lop_and_or(g1s, mf0, k6400),
             lop_and_or(h1s, mf0, k6400), xh.z, xh.w, acch);
    fold_d(tot, accl, s[0], s[2]);
    fold_d(tot + 4, acch, s[1], s[3]);
  }
}

// Q4_0: 8 blocks of 18 bytes (fp16 d + 16 nibble bytes; byte i: low nibble ->
// x[i], high -> x[16+i]); value d*(q-8), q entered as q*2^-24. Thread t takes
// bytes 4t..4t+3 of every block.
__device__ __forceinline__ void unit_q40(const UnitCtx& c, float* tot, float* cm) {
  const uint32_t m0f = 0x000F000Fu, k6400 = 0u;
  {
    const uint32_t o = 36u * c.t;  // blocks 2t, 2t+1
    const float2 cg = make_float2(8.f * half_bits_to_float(lds16(c.smem, c.rg + o)),
                                  8.f * half_bits_to_float(lds16(c.smem, c.rg + o + 18u)));
    const float2 cg8 = make_float2(8.f * half_bits_to_float(lds16(c.smem, c.rg8 + o)),
                                   8.f * half_bits_to_float(lds16(c.smem, c.rg8 + o + 18u)));
    coef_mma(c, cm, cg, cg8, make_float2(0.f, 0.f), make_float2(0.f, 0.f));
  }
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const uint32_t og = c.rg + 18u * b, og8 = c.rg8 + 18u * b;
    const float dg = 16777216.f * half_bits_to_float(lds16(c.smem, og));
    const float dg8 = 16777216.f * half_bits_to_float(lds16(c.smem, og8));
    const uint32_t wg = lds32_a2(c.smem, og + 2u + 4u * c.t), wg8 = lds32_a2(c.smem, og8 + 2u + 4u * c.t);
    const uint2 xl = ldx64(c, 32u * b + 4u * c.t);
    const uint2 xh = ldx64(c, 32u * b + 16u + 4u * c.t);
    const Nib4 a = nibbles(wg, m0f, k6400), a8 = nibbles(wg8, m0f, k6400);
    float acc[4];
    mma16816_z(acc, a.l02, a8.l02, a.l13, a8.l13, xl.x, xl.y);
    mma16816(acc, a.h02, a8.h02, a.h13, a8.h13, xh.x, xh.y, acc);
    fold_d(tot + 4 * (b & 1), acc, dg, dg8);
  }
}

// Q8_0: 8 blocks of 34 bytes (fp16 d + 32 int8); u = q+128 enters as u*2^-24,
// value d*q = d*u - 128 d. Thread t takes bytes 4t..4t+3 (k16 step 0) and
// 16+4t.. (step 1) of each block.
__device__ __forceinline__ void unit_q80(const UnitCtx& c, float* tot, float* cm) {
  const uint32_t mff = 0x00FF00FFu, kx = 0x00800080u;  // (w & 0x00FF00FF) ^ 0x00800080 = byte ^ 0x80
  {
    const uint32_t o = 68u * c.t;  // blocks 2t, 2t+1
    const float2 cg = make_float2(128.f * half_bits_to_float(lds16(c.smem, c.rg + o)),
                                  128.f * half_bits_to_float(lds16(c.smem, c.rg + o + 34u)));
    const float2 cg8 = make_float2(128.f * half_bits_to_float(lds16(c.smem, c.rg8 + o)),
                                   128.f * half_bits_to_float(lds16(c.smem, c.rg8 + o + 34u)));
    coef_mma(c, cm, cg, cg8, make_float2(0.f, 0.f), make_float2(0.f, 0.f));
  }
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const uint32_t og = c.rg + 34u * b, og8 = c.rg8 + 34u * b;
    const float dg = 16777216.f * half_bits_to_float(lds16(c.smem, og));
    const float dg8 = 16777216.f * half_bits_to_float(lds16(c.smem, og8));
    const uint32_t w0 = lds32_a2(c.smem, og + 2u + 4u * c.t), w1 = lds32_a2(c.smem, og + 18u + 4u * c.t);
    const uint32_t v0 = lds32_a2(c.smem, og8 + 2u + 4u * c.t), v1 = lds32_a2(c.smem, og8 + 18u + 4u * c.t);
    const uint2 x0 = ldx64(c, 32u * b + 4u * c.t);
    const uint2 x1 = ldx64(c, 32u * b + 16u + 4u * c.t);
    float acc[4];
    mma16816_z(acc, lop_and_xor(w0, mff, kx), lop_and_xor(v0, mff, kx), lop_and_xor(w0 >> 8, mff, kx),
               lop_and_xor(v0 >> 8, mff, kx), x0.x, x0.y);
    mma16816(acc, lop_and_xor(w1, mff, kx), lop_and_xor(v1, mff, kx), lop_and_xor(w1 >> 8, mff, kx),
             lop_and_xor(v1 >> 8, mff, kx), x1.x, x1.y, acc);
    fold_d(tot + 4 * (b & 1), acc, dg, dg8);
  }
}

// Q6_K: element e = 128h + 32u + cc (h = 0..1, u = 0..3, cc = 0..31):
// q6 = (ql[64h + 32(u&1) + cc] >> 4(u>>1)) & 15 | ((qh[128 + 32h + cc] >> 2u) & 3) << 4,
// value = (d * sc[e/16]) * (q6 - 32), q6 entered as q6*2^-24. One k16 step = one
// 16-weight scale group; thread t takes elements cc = 16s + 4t .. +3.
__device__ __forceinline__ void unit_q6k(const UnitCtx& c, float* tot, float* cm) {
  const uint32_t k6400 = 0u, m0f = 0x000F000Fu, m30 = 0x00300030u;
  const float dg = half_bits_to_float(lds16(c.smem, c.rg + 208u));
  const float dg8 = half_bits_to_float(lds16(c.smem, c.rg8 + 208u));
  {
    // groups 2t, 2t+1 (slots 2t, 2t+1) and 2t+8, 2t+9 (slots 2t+8, 2t+9)
    const uint32_t o = 192u + 2u * c.t;
    const uint32_t s0 = lds16(c.smem, c.rg + o), s1 = lds16(c.smem, c.rg + o + 8u);
    const uint32_t r0 = lds16(c.smem, c.rg8 + o), r1 = lds16(c.smem, c.rg8 + o + 8u);
    auto sc = [](uint32_t v, int i) { return static_cast<float>(static_cast<int8_t>(v >> (8 * i))); };
    const float kg = 32.f * dg, kg8 = 32.f * dg8;
    coef_mma(c, cm, make_float2(kg * sc(s0, 0), kg * sc(s0, 1)), make_float2(kg8 * sc(r0, 0), kg8 * sc(r0, 1)),
             make_float2(kg * sc(s1, 0), kg * sc(s1, 1)), make_float2(kg8 * sc(r1, 0), kg8 * sc(r1, 1)));
  }
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
      // bytes (0,2) and (1,3): nibble | hi2 << 4 = q6 as an fp16 subnormal (q6 * 2^-24)
      const uint32_t a0 = lop_and_or(lg, m0f, lop_and_or(hg << 4, m30, k6400));
      const uint32_t a2 = lop_and_or(lg >> 8, m0f, lop_and_or(hg >> 4, m30, k6400));
      const uint32_t a1 = lop_and_or(lg8, m0f, lop_and_or(hg8 << 4, m30, k6400));
      const uint32_t a3 = lop_and_or(lg8 >> 8, m0f, lop_and_or(hg8 >> 4, m30, k6400));
      const uint2 xb = ldx64(c, 32u * grp + cc);
      float acc[4];
      mma16816_z(acc, a0, a1, a2, a3, xb.x, xb.y);
      const float dl = 16777216.f * dg * static_cast<float>(static_cast<int8_t>(scg >> (8 * s)));
      const float dl8 = 16777216.f * dg8 * static_cast<float>(static_cast<int8_t>(scg8 >> (8 * s)));
      fold_d(tot + 4 * s, acc, dl, dl8);
    }
  }
}

template <int QT>
__device__ __forceinline__ void process_unit(const UnitCtx& c, float* tot, float* cm) {
  if (QT == kQ4_K) unit_q4k(c, tot, cm);
  else if (QT == kQ4_0) unit_q40(c, tot, cm);
  else if (QT == kQ8_0) unit_q80(c, tot, cm);
  else unit_q6k(c, tot, cm);
}

// ---- the kernel ---------------------------------------------------------------------
__device__ __forceinline__ const MmaSeg& seg_of(const MmaArgs& a, int64_t rb) {
  int i = 0;
#pragma unroll
  for (int j = 1; j < kMaxSegs; ++j)
    if (j < a.nseg && rb >= a.seg[j].rb0) i = j;
  return a.seg[i];
}

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
  __nv_bfloat16* xsb = reinterpret_cast<__nv_bfloat16*>(smem + a.xsb_off);  // [unit][col][t][4] hi, then lo
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

  // piece p -> (row block, chunk); 16 rows, one bulk copy per row into the padded stage
  const uint64_t wpol = l2_evict_first_policy();  // weights are read once per call
  auto issue = [&](int64_t p, int s) {
    const int64_t rb = blockIdx.x + (p / a.nchunks) * gridDim.x;
    const int ch = static_cast<int>(p % a.nchunks);
    const MmaSeg& sg = seg_of(a, rb);
    const int64_t r0 = (rb - sg.rb0) * kRowsPerBlock;
    const int nr = static_cast<int>((sg.n - r0) < kRowsPerBlock ? (sg.n - r0) : kRowsPerBlock);
    const int units = min(a.chunk_units, total_units - ch * a.chunk_units);
    const uint32_t bytes = static_cast<uint32_t>(units * a.unit_bytes);
    uint8_t* dst = smem + s * a.stage_bytes;
    const uint8_t* src = sg.q + r0 * a.row_bytes + static_cast<int64_t>(ch) * a.chunk_bytes;
    if (!a.lead) {
      mbar_arrive_expect_tx(&full[s], bytes * nr);
      for (int r = 0; r < nr; ++r) bulk_g2s_hint(dst + r * a.row_pitch, src + r * a.row_bytes, bytes, &full[s], wpol);
      return;
    }
    // Row starts are only 2-byte aligned: copy [start & ~15, end rounded up to 16) of
    // each row (the bytes around it belong to the neighbouring rows, inside the tensor).
    // The tensor's very last row ends where nothing may be read beyond it: its copy
    // stops at end & ~15 and the remaining < 16 bytes are plain loads, stored before
    // the arrive below (whose release makes them visible with the bulk bytes).
    const bool last_piece = r0 + nr == sg.n && ch == a.nchunks - 1;
    uint32_t tx = 0;
    for (int r = 0; r < nr; ++r) {
      const uintptr_t st = reinterpret_cast<uintptr_t>(src + r * a.row_bytes), en = st + bytes;
      const uintptr_t a0 = st & ~uintptr_t(15);
      const uintptr_t a1 = (last_piece && r == nr - 1) ? (en & ~uintptr_t(15)) : ((en + 15) & ~uintptr_t(15));
      tx += static_cast<uint32_t>(a1 - a0);
      if (last_piece && r == nr - 1) {
        uint8_t* d = dst + r * a.row_pitch + (a1 - a0);
        for (uintptr_t o = a1; o < en; o += 2)
          *reinterpret_cast<uint16_t*>(d + (o - a1)) = *reinterpret_cast<const uint16_t*>(o);
      }
    }
    mbar_arrive_expect_tx(&full[s], tx);
    for (int r = 0; r < nr; ++r) {
      const uintptr_t st = reinterpret_cast<uintptr_t>(src + r * a.row_bytes), en = st + bytes;
      const uintptr_t a0 = st & ~uintptr_t(15);
      const uintptr_t a1 = (last_piece && r == nr - 1) ? (en & ~uintptr_t(15)) : ((en + 15) & ~uintptr_t(15));
      bulk_g2s_hint(dst + r * a.row_pitch, reinterpret_cast<const void*>(a0), static_cast<uint32_t>(a1 - a0), &full[s],
                    wpol);
    }
  };
  __syncthreads();  // barriers initialised
  // Let the next kernel on the stream begin its own prologue as SMs free up.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == W) {
    // ---------------- producer ----------------
    // Weights are read-only inputs: the producer streams them from the start
    // and takes no part in staging x, so the issue back-pressure of the first
    // stages never holds up the other warps.
    if (lane == 0) {
      for (int64_t p = 0; p < total_pieces; ++p) {
        const int s = static_cast<int>(p % a.stages);
        if (p >= a.stages && !mbar_wait(&empty[s], static_cast<uint32_t>(((p / a.stages) - 1) & 1))) break;
        issue(p, s);
      }
    }
  } else {
  // The activations (and the outputs) may belong to the previous kernel: wait for it.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int stid = warp < W ? tid : tid - 32;  // staging threads: all but the producer warp

  // activations -> permuted fp16 [cols][k]; sums per 16 / 32 weights, [k/16][8] / [k/32][8]
  {
    const int groups = a.k / 8;  // 8 consecutive k per task
    const int nparts = a.xtype == GGUFMM_F32 ? 2 : 1;
    for (int task = stid; task < a.m * groups; task += kThreads - 32) {
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
        // x sums per scale group (16 weights = 2 tasks for Q6_K, 32 = 4 tasks otherwise),
        // stored as bf16 hi + lo in the B-fragment slot order of coef_mma:
        // slot j -> position 4 * ((j & 7) >> 1) + (j & 1) + 2 * (j >> 3)
        s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
        if (QT != kQ6_K) s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);
        const int gsz = QT == kQ6_K ? 16 : 32;
        if ((task & (gsz / 8 - 1)) == 0) {
          const int unit = k0 / kUnitK, j = (k0 % kUnitK) / gsz;
          __nv_bfloat16* e = xsb + (unit * a.cols + col) * 16;
          const __nv_bfloat16 hi = __float2bfloat16_rn(s);
          const __nv_bfloat16 lo = __float2bfloat16_rn(s - __bfloat162float(hi));
          const int pos = 4 * ((j & 7) >> 1) + (j & 1) + 2 * (j >> 3);
          e[pos] = hi;
          e[pos + a.xsb_lo / 2] = lo;
          if (QT != kQ6_K) {  // 8 groups per unit: slots 8..15 are zero
            e[pos + 2] = __float2bfloat16_rn(0.f);
            e[pos + 2 + a.xsb_lo / 2] = __float2bfloat16_rn(0.f);
          }
        }
      }
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kThreads - 32) : "memory");  // x staged (all but the producer)

  if (warp == W + 1) {
    // ---------------- epilogue ----------------
    for (int64_t blk = 0; blk < my_blocks; ++blk) {
      const int b = static_cast<int>(blk & 1);
      if (!mbar_wait(&rfull[b], static_cast<uint32_t>((blk >> 1) & 1))) break;
      const int64_t rb = blockIdx.x + blk * gridDim.x;
      const float* rbuf = red + b * (W * kRowsPerBlock * 8);
      const MmaSeg& sg = seg_of(a, rb);
      for (int i = lane; i < kRowsPerBlock * a.m; i += 32) {
        const int row = i / a.m, tok = i - row * a.m;
        const int64_t n_idx = (rb - sg.rb0) * kRowsPerBlock + row;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < W; ++w) {
          v += rbuf[(w * kRowsPerBlock + row) * 8 + tok];
          if (a.cols > a.m) v += rbuf[(w * kRowsPerBlock + row) * 8 + tok + a.m];
        }
        if (n_idx < sg.n) store_y_rt(sg.y, a.ytype, tok * sg.ldy + n_idx, v);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&rempty[b]);
    }
  } else {
    // ---------------- compute ----------------
    const uint32_t xcol = a.x_off + (g < a.cols ? g : 0) * a.x_pitch;
    const int gcol = g < a.cols ? g : 0;
    float tot[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // two independent fold chains
    float tot2[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // ... for the second unit of a pair
    float cm[4] = {0.f, 0.f, 0.f, 0.f};                         // bias / min terms (coef_mma)
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
        uint32_t lead_g = 0, lead_g8 = 0;  // where rows g, g+8 start inside their slots
        if (a.lead) {
          const int64_t rb = blockIdx.x + blk * gridDim.x;
          const MmaSeg& sg = seg_of(a, rb);
          const int64_t off = ((rb - sg.rb0) * kRowsPerBlock + g) * a.row_bytes + static_cast<int64_t>(ch) * a.chunk_bytes;
          lead_g = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(sg.q) + off) & 15);
          lead_g8 = static_cast<uint32_t>((reinterpret_cast<uintptr_t>(sg.q) + off + 8 * a.row_bytes) & 15);
        }
        auto ctx = [&](int u) {
          const int ku = (ch * a.chunk_units + u) * kUnitK;
          UnitCtx c;
          c.smem = smem;
          c.rg = sbase + lead_g + u * a.unit_bytes;
          c.rg8 = sbase + 8 * a.row_pitch + lead_g8 + u * a.unit_bytes;
          c.xo = xcol + 2u * ku;
          c.xsh = a.xsb_off + static_cast<uint32_t>((((ku / kUnitK) * a.cols + gcol) * 4 + t) * 8);
          c.xsl_add = a.xsb_lo;
          c.t = t;
          c.lane = lane;
          return c;
        };
        int u = warp;
        // two units at a time, in straight-line code with separate accumulators,
        // so the loads and MMAs of one overlap the dependency chains of the other
        for (; u + W < units; u += 2 * W) {
          const UnitCtx c0 = ctx(u), c1 = ctx(u + W);
          process_unit<QT>(c0, tot, cm);
          process_unit<QT>(c1, tot2, cm);
        }
        if (u < units) process_unit<QT>(ctx(u), tot, cm);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with stage s
      }
      if (!ok) break;
      // row block complete: park the partial 16 x 8 tile for the epilogue
      const int b = static_cast<int>(blk & 1);
      if (blk >= kRedBufs && !mbar_wait(&rempty[b], static_cast<uint32_t>(((blk >> 1) - 1) & 1))) break;
      float* rw = red + b * (W * kRowsPerBlock * 8) + warp * (kRowsPerBlock * 8);
#pragma unroll
      for (int i = 0; i < 8; ++i) tot[i] += tot2[i];
      *reinterpret_cast<float2*>(rw + g * 8 + 2 * t) =
          make_float2(tot[0] + tot[4] - cm[0], tot[1] + tot[5] - cm[1]);
      *reinterpret_cast<float2*>(rw + (g + 8) * 8 + 2 * t) =
          make_float2(tot[2] + tot[6] - cm[2], tot[3] + tot[7] - cm[3]);
#pragma unroll
      for (int i = 0; i < 8; ++i) tot[i] = tot2[i] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; ++i) cm[i] = 0.f;
      __syncwarp();
      if (lane == 0) mbar_arrive(&rfull[b]);
    }
  }
  }  // not the producer
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

// Compute warps per CTA (8 by default; GGUFMM_GEMV_F16_WARPS=4 for tuning).
static int compute_warps() {
  static const int w = [] {
    const char* e = std::getenv("GGUFMM_GEMV_F16_WARPS");
    const int v = e ? std::atoi(e) : 8;
    return v == 4 ? 4 : 8;
  }();
  return w;
}

// Whether the tensor-core GEMV handles this problem; fills the launch plan.
static bool plan_mma(int qt, int64_t k, int m, int xtype, int smem_budget, int W, MmaArgs& a) {
  a.unit_bytes = unit_bytes_of(qt);
  if (!a.unit_bytes || k % kUnitK || m < 1 || m > 8) return false;
  a.cols = xtype == GGUFMM_F32 ? 2 * m : m;
  if (a.cols > 8) return false;
  const int units = static_cast<int>(k / kUnitK);
  // Q6_K superblocks are 210 bytes: rows are 16-byte multiples only when K/256 is a
  // multiple of 8; otherwise every row's copy starts at its aligned-down address
  // (a.lead) and its slot holds up to 15 bytes more. Chunks of 8 / 16 units stay
  // 16-byte multiples, so only the row start moves.
  a.lead = qt == kQ6_K && units % 8 != 0;
  a.chunk_units = std::min(units, kMaxChunkUnits);
  if (qt == kQ6_K && a.chunk_units >= 8) a.chunk_units -= a.chunk_units % 8;
  a.nchunks = (units + a.chunk_units - 1) / a.chunk_units;
  a.chunk_bytes = a.chunk_units * a.unit_bytes;
  if (a.chunk_bytes % 16 && !(a.lead && a.nchunks == 1)) return false;
  // pitch = 32 mod 128: conflict-free 8-byte row reads (+16 for the aligned-down start)
  a.row_pitch = (a.chunk_bytes + (a.lead ? 16 : 0) + 127) / 128 * 128 + 32;
  a.stage_bytes = kRowsPerBlock * a.row_pitch;
  a.x_pitch = static_cast<int>(2 * k + 64);
  const int x_bytes = a.cols * a.x_pitch;
  const int xsb_half = static_cast<int>(k / kUnitK) * a.cols * 32;  // 16 bf16 slots per (unit, column)
  const int red_bytes = kRedBufs * W * kRowsPerBlock * 8 * 4;
  const int fixed = x_bytes + 2 * xsb_half + red_bytes + 16 * 8 + 64;
  const int stages = std::min(6, (smem_budget - fixed) / a.stage_bytes);
  if (stages < 2) return false;
  a.stages = stages;
  a.x_off = static_cast<uint32_t>(stages * a.stage_bytes);
  a.xsb_off = a.x_off + x_bytes;
  a.xsb_lo = static_cast<uint32_t>(xsb_half);
  a.red_off = a.xsb_off + 2 * xsb_half;
  a.bar_off = (a.red_off + red_bytes + 7) / 8 * 8;
  return true;
}

bool gemv_mma_supported(int qtype, int64_t n, int64_t k, int m, int xtype) {
  MmaArgs a{};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const DevInfo di = device_info(dev);
  (void)n;
  return plan_mma(qtype, k, m, xtype, std::min(di.smem_optin, 227 * 1024), compute_warps(), a);
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
  // programmatic dependent launch: this kernel's weight prefetch may overlap the
  // tail of the previous kernel on the stream (it waits before touching x / y)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3((W + 2) * 32);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, a);
}

template <int QT>
static cudaError_t launch_mma_q(MmaArgs& a, int W, int dev, const DevInfo& di, cudaStream_t st) {
  if (W == 4) return launch_mma_t<QT, 4>(a, dev, di, st);
  return launch_mma_t<QT, 8>(a, dev, di, st);
}

// nseg weights of the same qtype and K (each 16-byte aligned, row bytes a
// multiple of 16) against the same activations, one launch.
cudaError_t launch_gemv_mma_grouped(int nseg, const void* const* q, const int64_t* n, int qtype, int64_t k,
                                    const void* x, int xtype, int64_t m, int64_t ldx, void* const* y, int ytype,
                                    const int64_t* ldy, int64_t row_bytes, cudaStream_t st) {
  if (nseg < 1 || nseg > kMaxSegs) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const DevInfo di = device_info(dev);
  const int W = compute_warps();
  MmaArgs a{};
  if (!plan_mma(qtype, k, static_cast<int>(m), xtype, std::min(di.smem_optin, 227 * 1024), W, a))
    return cudaErrorInvalidValue;
  a.nseg = nseg;
  int64_t rb = 0;
  for (int i = 0; i < nseg; ++i) {
    a.seg[i].q = static_cast<const uint8_t*>(q[i]);
    a.seg[i].y = y[i];
    a.seg[i].n = n[i];
    a.seg[i].ldy = ldy[i];
    a.seg[i].rb0 = rb;
    rb += (n[i] + kRowsPerBlock - 1) / kRowsPerBlock;
  }
  a.nrowblocks = rb;
  a.k = static_cast<int>(k);
  a.row_bytes = row_bytes;
  a.x = x;
  a.xtype = xtype;
  a.ldx = ldx;
  a.m = static_cast<int>(m);
  a.ytype = ytype;
  switch (qtype) {
    case kQ4_K: return launch_mma_q<kQ4_K>(a, W, dev, di, st);
    case kQ4_0: return launch_mma_q<kQ4_0>(a, W, dev, di, st);
    case kQ8_0: return launch_mma_q<kQ8_0>(a, W, dev, di, st);
    case kQ6_K: return launch_mma_q<kQ6_K>(a, W, dev, di, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv_mma(const void* q, int qtype, int64_t n, int64_t k, const void* x, int xtype, int64_t m,
                            int64_t ldx, void* y, int ytype, int64_t ldy, int64_t row_bytes, cudaStream_t st) {
  return launch_gemv_mma_grouped(1, &q, &n, qtype, k, x, xtype, m, ldx, &y, ytype, &ldy, row_bytes, st);
}

cudaError_t gemv_mma_device_error(int* v, int clear, cudaStream_t st) { return tu_device_error(v, clear, st); }
cudaError_t gemv_mma_set_wait_limit(uint32_t polls) { return tu_set_wait_limit(polls); }

}  // namespace ggufmm
