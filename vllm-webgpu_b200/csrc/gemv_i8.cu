// gemv_i8.cu -- decode GEMV (M <= 8 tokens) for Q4_K and Q4_0 on the integer
// tensor-core path (mma.sync m16n8k32, u8 weights x s8 activation digits,
// s32 accumulation), straight from GGUF blocks.
//
//   y[m, n] = sum_k x[m, k] W[n, k]
//
// Why integers: at HBM speed the cost of a 4-bit GEMV is the per-weight decode,
// and on the u8 path a 4-bit quant is ready for the MMA after ONE lop3 per FOUR
// weights (w & 0x0F0F0F0F are four u8 quants; Q4_K high nibbles are used in
// place, w & 0xF0F0F0F0 = 16 q). One m16n8k32 consumes 512 weights.
//
// Activations as exact integer digits: every 256 consecutive activations of a
// token (one K-quant superblock, 8 Q4_0 blocks) get a power-of-two scale s with
// max|x| / s in [2^21, 2^22), and X = rint(x / s) is written as three balanced
// signed bytes, X = 65536 d1 + 256 d2 + d3. Each digit is one B column of the
// MMA (the n8 tile holds the 3 digits of up to 2 tokens for free), so the MMA
// result is exact and the only rounding of x is rint at 2^-22 of the group
// maximum (fp32-like; bf16 / fp16 inputs are mostly exact).
//
// Scales, exactly:
//   Q4_K  value = d sc_j q - dmin m_j (j = 32-weight sub-block). Per unit the
//         integer sum T = sum_j sc_j * acc_j is formed with integer multiply-adds
//         (acc_j = one MMA, highs carry the factor 16 and lows get it at the
//         end), converted once and folded with (d / 16) * s * radix. The min
//         part dmin * sum_j m_j X_j runs as a bf16 MMA with the exact 6-bit m_j
//         against the per-sub-block sums of x (bf16 hi + lo).
//   Q4_0  value = d (q - 8): the MMA's C operand carries -8 * sum(digits of the
//         block), so each block's accumulator is sum (q - 8) X exactly; folded
//         with the block's fp16 d.
// Precision is therefore that of fp32 arithmetic on the exact dequantized
// weights (the reference's dequantize-then-matmul), not an fp16 weight.
//
// Pipeline: one producer warp streams pieces (16 rows x up to 32 units of 256
// weights) into a shared-memory ring with 1-D bulk copies of >= 4 KB where the
// layout allows (several whole rows per copy: short copies are request-bound);
// W compute warps take every W-th unit; one epilogue warp sums the warps'
// partials of a row block and writes y. The producer takes no part in staging
// x, so its copy back-pressure never stalls the other warps. Bounded mbarrier
// waits throughout.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"

namespace ggufmm {

namespace {

constexpr int kRows = 16;
constexpr int kUnitK = 256;
constexpr int kCopyBytes = 4608;  // target bytes per bulk copy
constexpr int kRedBufs = 2;
constexpr int kMaxSegs = 4;

struct Seg {
  const uint8_t* q;
  void* y;
  int64_t n;
  int64_t ldy;
  int64_t rb0;
};

struct I8Args {
  Seg seg[kMaxSegs];
  int nseg;
  int k;
  int64_t row_bytes;
  const void* x;
  int xtype;
  int64_t ldx;
  int m;
  int ytype;
  int unit_bytes;
  int chunk_units;
  int nchunks;
  int chunk_bytes;
  int rg;            // rows per bulk copy (several whole rows when one chunk spans the row)
  int group_pitch;   // smem bytes per copied row group (32 mod 128)
  int stage_bytes;
  int stages;
  int64_t nrowblocks;
  int xd_pitch;      // bytes per digit column of x
  int red_stride;    // floats per warp in one reduction buffer
  int ksplit;        // 1, or 2: K halves on the two CTAs of a cluster, partials joined in rank 0
  int swiglu;        // segments 0 (gate) and 1 (up) of equal N: y = silu(gate) * up into segment 0's y
  const void* resid; // optional residual added to segment 0's y (y's dtype, row stride ldr; may alias y)
  int64_t ldr;
  // all-reduce over tp_world GPUs through peer memory (tp_world > 1): every GPU's
  // exchange buffer, [kTpHdr bytes: u32 generation per CTA][2 parities][tp_world
  // sources][m_max][n] 8-byte words (generation << 32 | fp32 partial); y = the sum of
  // the partials
  int tp_world, tp_rank;
  uint32_t epoch;
  int64_t m_max, tp_nrb, tp_flag_off;  // flag_off in bytes
  uint64_t peer[8];
  uint32_t xd_off;   // int8 digits [3m cols][k]
  uint32_t xf_off;   // float fold factors [unit][8 NCG cols]: s * radix
  uint32_t xs_off;   // Q4_K: bf16 x sums [unit][8 NCC cols][8 sub-blocks]; Q4_0: int -8*digit sums [block][8 NCG cols]
  uint32_t red_off;
  uint32_t xchg_off;  // ksplit 2: [2 slots][8 tokens][16 rows] floats of rank 1's partials, in rank 0
  uint32_t bar_off;
};

// ---- cluster (distributed shared memory) helpers for the K split ----
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
  const uint32_t lim = g_wait_limit;
  for (uint32_t i = 0; i < lim; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    if (i > 256) __nanosleep(64);
  }
  atomicOr(&g_device_error, kErrWaitTimeout);
  return false;
}
// ---- peer-memory (NVLink) exchange for the fused all-reduce ----
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
constexpr int64_t kTpHdr = 4096;  // u32 generation per CTA (at most 1024 CTAs)

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void imma(int* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                     uint32_t b1, int c0, int c1, int c2, int c3) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(c0), "r"(c1), "r"(c2), "r"(c3));
}

__device__ __forceinline__ void mma_bf16_z(float* d, uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(0u), "r"(0u), "r"(b0), "r"(0u), "f"(0.f));
}

template <typename T>
__device__ __forceinline__ T lds(const uint8_t* smem, uint32_t off) {
  return *reinterpret_cast<const T*>(smem + off);
}

// 4 bytes at a 2-byte aligned offset.
__device__ __forceinline__ uint32_t lds32_a2(const uint8_t* smem, uint32_t off) {
  const uint32_t* w = reinterpret_cast<const uint32_t*>(smem + (off & ~3u));
  return __funnelshift_r(w[0], w[1], (off & 3u) * 8u);
}

__device__ __forceinline__ uint32_t byte_of(uint32_t w, int i) { return __byte_perm(w, 0u, 0x4440u | i); }

// bf16 bits of a small non-negative integer (exact), packed as (lo, hi).
__device__ __forceinline__ uint32_t bf16x2_of_small(uint32_t lo, uint32_t hi) {
  const uint32_t fl = __float_as_uint(static_cast<float>(lo)), fh = __float_as_uint(static_cast<float>(hi));
  return __byte_perm(fl, fh, 0x7632u);
}

struct Ctx {
  const uint8_t* smem;
  uint32_t rg, rg8;  // unit's bytes in the weight rows of MMA rows g, g+8
  uint32_t xo[3];    // digit column (per col group) + unit's first k + 8t
  uint32_t xf;       // fold factors of this unit, cols 2t, 2t+1 of col group 0
  uint32_t xs;       // Q4_K: x-sum word (unit, coef col g, t); Q4_0: C words of the unit's block 0
  int t;
};

// ---- Q4_K: 8 sub-blocks of 32; chunk c = qs bytes 32c..32c+31, low nibbles ->
// sub-block 2c, high -> 2c+1. Thread t takes bytes 8t..8t+7 of a chunk: A regs
// (row g / g+8) x (bytes 8t..8t+3 = MMA k 4t..4t+3, bytes 8t+4..8t+7 = k 16+4t..),
// matching digits stored in natural k order.
template <int NCG, int NCC>
__device__ __forceinline__ void unit_q4k(const Ctx& c, float (&ft)[NCG][4], float (&cmin)[2 * NCC]) {
  const uint4 hg = lds<uint4>(c.smem, c.rg), hg8 = lds<uint4>(c.smem, c.rg8);
  uint32_t scl[2], sch[2];
  float dd[2], dm[2];
  uint32_t ma[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const uint4 h = r == 0 ? hg : hg8;
    dd[r] = half_bits_to_float(h.x) * 0.0625f;
    dm[r] = half_bits_to_float(h.x >> 16);
    // 6-bit scales / mins (gguf quants.py:479-501): sub-blocks 0..3 from bytes 0..3 / 4..7,
    // 4..7 from the low / high nibbles of bytes 8..11 plus the top bits of bytes 0..7
    scl[r] = h.y & 0x3F3F3F3Fu;
    sch[r] = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t ml = h.z & 0x3F3F3F3Fu;
    const uint32_t mh = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
    const uint32_t mw = c.t < 2 ? ml : mh;  // this thread's slots: sub-blocks 2t, 2t+1
    const int b0 = 2 * (c.t & 1);
    ma[r] = bf16x2_of_small(byte_of(mw, b0), byte_of(mw, b0 + 1));
  }
  // min part: sum_j m_j * xsum_j, cols (token, hi / lo)
#pragma unroll
  for (int cc = 0; cc < NCC; ++cc) {
    float am[4];
    mma_bf16_z(am, ma[0], ma[1], lds<uint32_t>(c.smem, c.xs + cc * 8 * 16));
    cmin[2 * cc] = fmaf(dm[0], am[0] + am[1], cmin[2 * cc]);
    cmin[2 * cc + 1] = fmaf(dm[1], am[2] + am[3], cmin[2 * cc + 1]);
  }
  int tl[NCG][4], th[NCG][4];
#pragma unroll
  for (int ch = 0; ch < 4; ++ch) {
    const uint2 w = lds<uint2>(c.smem, c.rg + 16u + 32u * ch + 8u * c.t);
    const uint2 w8 = lds<uint2>(c.smem, c.rg8 + 16u + 32u * ch + 8u * c.t);
    const uint32_t m0f = 0x0F0F0F0Fu, mf0 = 0xF0F0F0F0u;
    const uint32_t l0 = w.x & m0f, l1 = w8.x & m0f, l2 = w.y & m0f, l3 = w8.y & m0f;
    const uint32_t h0 = w.x & mf0, h1 = w8.x & mf0, h2 = w.y & mf0, h3 = w8.y & mf0;
    // sub-blocks 2ch (lows) and 2ch+1 (highs): bytes of scl (ch < 2) or sch
    const uint32_t sw = ch < 2 ? scl[0] : sch[0], sw8 = ch < 2 ? scl[1] : sch[1];
    const int bl = 2 * (ch & 1);
    const int sl = static_cast<int>(byte_of(sw, bl)), sl8 = static_cast<int>(byte_of(sw8, bl));
    const int sh = static_cast<int>(byte_of(sw, bl + 1)), sh8 = static_cast<int>(byte_of(sw8, bl + 1));
#pragma unroll
    for (int cg = 0; cg < NCG; ++cg) {
      const uint2 xl = lds<uint2>(c.smem, c.xo[cg] + 64u * ch);
      const uint2 xh = lds<uint2>(c.smem, c.xo[cg] + 64u * ch + 32u);
      int al[4], ah[4];
      imma(al, l0, l1, l2, l3, xl.x, xl.y, 0, 0, 0, 0);
      imma(ah, h0, h1, h2, h3, xh.x, xh.y, 0, 0, 0, 0);
      if (ch == 0) {
        tl[cg][0] = sl * al[0]; tl[cg][1] = sl * al[1]; tl[cg][2] = sl8 * al[2]; tl[cg][3] = sl8 * al[3];
        th[cg][0] = sh * ah[0]; th[cg][1] = sh * ah[1]; th[cg][2] = sh8 * ah[2]; th[cg][3] = sh8 * ah[3];
      } else {
        tl[cg][0] += sl * al[0]; tl[cg][1] += sl * al[1]; tl[cg][2] += sl8 * al[2]; tl[cg][3] += sl8 * al[3];
        th[cg][0] += sh * ah[0]; th[cg][1] += sh * ah[1]; th[cg][2] += sh8 * ah[2]; th[cg][3] += sh8 * ah[3];
      }
    }
  }
  // lows carry q, highs 16 q: unit sum = (d / 16) * (16 tl + th); |16 tl + th| < 2^29
#pragma unroll
  for (int cg = 0; cg < NCG; ++cg) {
    const float2 f = lds<float2>(c.smem, c.xf + cg * 32u);
    ft[cg][0] = fmaf(dd[0] * f.x, static_cast<float>(16 * tl[cg][0] + th[cg][0]), ft[cg][0]);
    ft[cg][1] = fmaf(dd[0] * f.y, static_cast<float>(16 * tl[cg][1] + th[cg][1]), ft[cg][1]);
    ft[cg][2] = fmaf(dd[1] * f.x, static_cast<float>(16 * tl[cg][2] + th[cg][2]), ft[cg][2]);
    ft[cg][3] = fmaf(dd[1] * f.y, static_cast<float>(16 * tl[cg][3] + th[cg][3]), ft[cg][3]);
  }
}

// ---- Q4_0: 8 blocks of 18 bytes (fp16 d + 16 nibble bytes; byte i: low -> x[i],
// high -> x[16+i]). Thread t takes bytes 4t..4t+3 of a block: lows are MMA k
// 4t..4t+3, highs k 16+4t..; the digits of a block are stored permuted so both
// halves are one 8-byte load. C = -8 * (digit sums of the block, per column).
template <int NCG>
__device__ __forceinline__ void unit_q40(const Ctx& c, float (&ft)[NCG][4]) {
  float fb[NCG][4];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const uint32_t og = c.rg + 18u * b, og8 = c.rg8 + 18u * b;
    const float dg = half_bits_to_float(lds<uint16_t>(c.smem, og));
    const float dg8 = half_bits_to_float(lds<uint16_t>(c.smem, og8));
    // block b starts at 18b: its nibbles at 18b + 2 + 4t are 4-byte aligned for odd b
    uint32_t w, w8;
    if (b & 1) {
      w = lds<uint32_t>(c.smem, og + 2u + 4u * c.t);
      w8 = lds<uint32_t>(c.smem, og8 + 2u + 4u * c.t);
    } else {
      w = lds32_a2(c.smem, og + 2u + 4u * c.t);
      w8 = lds32_a2(c.smem, og8 + 2u + 4u * c.t);
    }
    const uint32_t m0f = 0x0F0F0F0Fu;
    const uint32_t a0 = w & m0f, a1 = w8 & m0f, a2 = (w >> 4) & m0f, a3 = (w8 >> 4) & m0f;
#pragma unroll
    for (int cg = 0; cg < NCG; ++cg) {
      const uint2 xb = lds<uint2>(c.smem, c.xo[cg] + 32u * b);
      const int2 cn = lds<int2>(c.smem, c.xs + (b * NCG + cg) * 32u);
      int acc[4];
      imma(acc, a0, a1, a2, a3, xb.x, xb.y, cn.x, cn.y, cn.x, cn.y);
      if (b == 0) {
        fb[cg][0] = dg * static_cast<float>(acc[0]);
        fb[cg][1] = dg * static_cast<float>(acc[1]);
        fb[cg][2] = dg8 * static_cast<float>(acc[2]);
        fb[cg][3] = dg8 * static_cast<float>(acc[3]);
      } else {
        fb[cg][0] = fmaf(dg, static_cast<float>(acc[0]), fb[cg][0]);
        fb[cg][1] = fmaf(dg, static_cast<float>(acc[1]), fb[cg][1]);
        fb[cg][2] = fmaf(dg8, static_cast<float>(acc[2]), fb[cg][2]);
        fb[cg][3] = fmaf(dg8, static_cast<float>(acc[3]), fb[cg][3]);
      }
    }
  }
#pragma unroll
  for (int cg = 0; cg < NCG; ++cg) {
    const float2 f = lds<float2>(c.smem, c.xf + cg * 32u);
    ft[cg][0] = fmaf(f.x, fb[cg][0], ft[cg][0]);
    ft[cg][1] = fmaf(f.y, fb[cg][1], ft[cg][1]);
    ft[cg][2] = fmaf(f.x, fb[cg][2], ft[cg][2]);
    ft[cg][3] = fmaf(f.y, fb[cg][3], ft[cg][3]);
  }
}

// MMA row mr (0..15) of a row block <-> weight row: with rg rows per copy the
// row groups sit at group_pitch = 32 mod 128, and MMA rows 0..7 (one A register
// each) take the first row of distinct groups where possible, so the 8-byte
// reads of a quarter warp fall in distinct banks.
__device__ __forceinline__ int phys_row(int mr, int rg) {
  const int per = kRows / rg;
  return rg * (mr % per) + mr / per;
}
__device__ __forceinline__ uint32_t row_off(int pr, const I8Args& a) {
  return static_cast<uint32_t>((pr / a.rg) * a.group_pitch + (pr % a.rg) * a.chunk_bytes);
}

__device__ __forceinline__ const Seg& seg_of(const I8Args& a, int64_t rb) {
  int i = 0;
#pragma unroll
  for (int j = 1; j < kMaxSegs; ++j)
    if (j < a.nseg && rb >= a.seg[j].rb0) i = j;
  return a.seg[i];
}

// The j-th row block of cluster / CTA `cid`: plain, every ncl-th block; SwiGLU,
// every ncl-th PAIR of blocks (gate rows, then the same up rows), so the epilogue
// holds the gate sums when the up sums arrive.
template <bool EXT>
__device__ __forceinline__ int64_t block_of(const I8Args& a, int64_t cid, int64_t ncl, int64_t j) {
  return EXT && a.swiglu ? 2 * (cid + (j >> 1) * ncl) + (j & 1) : cid + j * ncl;
}
// Segment and first weight row of logical row block lb.
template <bool EXT>
__device__ __forceinline__ const Seg& block_rows(const I8Args& a, int64_t lb, int64_t& r0) {
  if (EXT && a.swiglu) {
    r0 = (lb >> 1) * kRows;
    return a.seg[lb & 1];
  }
  const Seg& sg = seg_of(a, lb);
  r0 = (lb - sg.rb0) * kRows;
  return sg;
}

// Position of element e (0..31) of a Q4_0 block inside its 32 permuted digit
// bytes: thread t's MMA k 4t..4t+3 (elements 4t..) and 16+4t.. (elements 16+4t..)
// become bytes 8t..8t+7.
__device__ __forceinline__ int q40_pos(int e) { return e < 16 ? (e >> 2) * 8 + (e & 3) : ((e - 16) >> 2) * 8 + 4 + (e & 3); }

// EXT: the SwiGLU / all-reduce epilogue variants (plain GEMVs compile without them)
// MINB: CTAs per SM the launch is shaped for (registers are capped to fit them).
template <int QT, int NCG, int NCC, int W, bool EXT, int MINB>
__global__ void __launch_bounds__((W + 2) * 32, MINB) gemv_i8_kernel(const I8Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.bar_off);
  uint64_t* empty = full + a.stages;
  uint64_t* rfull = empty + a.stages;
  uint64_t* rempty = rfull + kRedBufs;
  uint64_t* xfull = rempty + kRedBufs;  // ksplit 2, rank 0: rank 1's partials of a slot have landed
  uint64_t* xempty = xfull + 2;         // ksplit 2, rank 1: rank 0 has consumed a slot
  float* red = reinterpret_cast<float*>(smem + a.red_off);
  // with the K split, the two CTAs of a cluster (consecutive blockIdx.x) share row blocks
  const int rank = a.ksplit == 2 ? static_cast<int>(blockIdx.x & 1) : 0;
  const int64_t cid = blockIdx.x / a.ksplit, ncl = gridDim.x / a.ksplit;
  const bool pairs = EXT && a.swiglu;
  const int64_t nunits = pairs ? a.nrowblocks / 2 : a.nrowblocks;  // blocks, or gate/up pairs
  const int64_t my_blocks = (nunits > cid ? (nunits - 1 - cid) / ncl + 1 : 0) * (pairs ? 2 : 1);
  const int64_t total_pieces = my_blocks * a.nchunks;
  const int units = a.k / kUnitK / a.ksplit;  // this CTA's units along K
  const int ku0 = rank * units;                // ... starting here
  constexpr int kDCols = 8 * NCG;  // digit columns (padded)
  constexpr int kCCols = 8 * NCC;  // Q4_K coef columns (token, hi / lo), padded

  if (tid == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], W);
    }
    for (int b = 0; b < kRedBufs; ++b) {
      mbar_init(&rfull[b], W);
      mbar_init(&rempty[b], 1);
    }
    mbar_init(&xfull[0], 1);
    mbar_init(&xfull[1], 1);
    mbar_init(&xempty[0], 1);
    mbar_init(&xempty[1], 1);
    fence_mbar_init();
  }

  const uint64_t wpol = l2_evict_first_policy();  // weights are read once per call
  auto issue = [&](int64_t p, int s) {
    const int64_t rb = block_of<EXT>(a, cid, ncl, p / a.nchunks);
    const int ch = static_cast<int>(p % a.nchunks);
    int64_t r0;
    const Seg& sg = block_rows<EXT>(a, rb, r0);
    const int nr = static_cast<int>((sg.n - r0) < kRows ? (sg.n - r0) : kRows);
    const int nu = min(a.chunk_units, units - ch * a.chunk_units);
    const uint32_t bytes = static_cast<uint32_t>(nu * a.unit_bytes);
    mbar_arrive_expect_tx(&full[s], bytes * nr);
    uint8_t* dst = smem + s * a.stage_bytes;
    const uint8_t* src = sg.q + r0 * a.row_bytes + static_cast<int64_t>(ku0) * a.unit_bytes +
                         static_cast<int64_t>(ch) * a.chunk_bytes;
    // rg > 1 only when a chunk is the whole row (one chunk, no K split): rg consecutive rows are contiguous
    for (int r = 0, grp = 0; r < nr; r += a.rg, ++grp) {
      const uint32_t rows = static_cast<uint32_t>(min(a.rg, nr - r));
      bulk_g2s_hint(dst + grp * a.group_pitch, src + r * a.row_bytes, rows * bytes, &full[s], wpol);
    }
  };

  __syncthreads();  // barriers initialised
  if (a.ksplit == 2) cluster_sync_all();  // ... in both CTAs of the cluster before any remote arrive
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == W) {
    // ---------------- producer ----------------
    // Weights are read-only: streamed from the start (under programmatic
    // dependent launch, before the previous kernel has finished). The producer
    // takes no part in staging x, so the back-pressure of its copies never holds
    // up the other warps.
    if (lane == 0) {
      for (int64_t p = 0; p < total_pieces; ++p) {
        const int s = static_cast<int>(p % a.stages);
        if (p >= a.stages && !mbar_wait(&empty[s], static_cast<uint32_t>(((p / a.stages) - 1) & 1))) break;
        issue(p, s);
      }
    }
  } else {
    // x and y may belong to the previous kernel on the stream
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // ---- activations -> digits. One warp per (token, unit): lane l holds x[8l..8l+7].
    // kB tasks of a warp go through each step together (step-major, straight-line
    // code), so their load round trips and reduction chains overlap.
    constexpr int kStagers = W + 1, kB = W == 8 && MINB == 1 ? 8 : 4;
    const int ntask = a.m * units;
    for (int base = warp < W ? warp : W; base < ntask; base += kB * kStagers) {
      int tok[kB], un[kB];
      bool valid[kB];
      uint4 raw[kB][2];
#pragma unroll
      for (int bt = 0; bt < kB; ++bt) {
        const int task = base + bt * kStagers;
        valid[bt] = task < ntask;
        const int tc = valid[bt] ? task : base;
        tok[bt] = tc / units;
        un[bt] = tc - tok[bt] * units;
        const int64_t k0 = static_cast<int64_t>(ku0 + un[bt]) * kUnitK + 8 * lane;
        if (a.xtype == GGUFMM_F32) {
          const uint4* xp = reinterpret_cast<const uint4*>(static_cast<const float*>(a.x) + tok[bt] * a.ldx + k0);
          raw[bt][0] = xp[0];
          raw[bt][1] = xp[1];
        } else {
          raw[bt][0] = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.x) + tok[bt] * a.ldx + k0);
        }
      }
      float v[kB][8];
      uint32_t mxb[kB];
#pragma unroll
      for (int bt = 0; bt < kB; ++bt) {
        if (a.xtype == GGUFMM_F32) {
          const uint32_t w8[8] = {raw[bt][0].x, raw[bt][0].y, raw[bt][0].z, raw[bt][0].w,
                                  raw[bt][1].x, raw[bt][1].y, raw[bt][1].z, raw[bt][1].w};
#pragma unroll
          for (int i = 0; i < 8; ++i) v[bt][i] = __uint_as_float(w8[i]);
        } else {
          const uint32_t w4[4] = {raw[bt][0].x, raw[bt][0].y, raw[bt][0].z, raw[bt][0].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (a.xtype == GGUFMM_BF16) {
              v[bt][2 * i] = __uint_as_float(w4[i] << 16);
              v[bt][2 * i + 1] = __uint_as_float(w4[i] & 0xFFFF0000u);
            } else {
              const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
              v[bt][2 * i] = f.x;
              v[bt][2 * i + 1] = f.y;
            }
          }
        }
        float mx = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) mx = fmaxf(mx, fabsf(v[bt][i]));
        // non-negative floats order like their bit patterns: one warp max
        mxb[bt] = __reduce_max_sync(0xFFFFFFFFu, __float_as_uint(mx));
      }
#pragma unroll
      for (int bt = 0; bt < kB; ++bt) {
        // max in [2^(E-127), 2^(E-126)): inv = 2^(148-E) puts it in [2^21, 2^22); groups
        // whose maximum is below 2^-105 (or zero) become zeros
        const uint32_t E = (mxb[bt] >> 23) & 0xFFu;
        const bool live = E >= 22u && E < 255u;
        const float inv = live ? __uint_as_float((275u - E) << 23) : 0.f;
        const float s = live ? __uint_as_float((E - 21u) << 23) : 0.f;
        // Balanced digits in one add: Y = X + 0x808080 (>= 0 as |X| <= 2^22) has the
        // bytes d3 + 128, d2 + 128, d1 + 128, so Y ^ 0x808080 holds d3, d2, d1 as s8.
        // rint(x * inv) without a float->int conversion: x * inv + 1.5 * 2^23 stays in
        // [2^23, 2^24), so its bit pattern is 0x4B400000 + X (rounded to nearest even)
        uint32_t z[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          z[i] = (__float_as_uint(fmaf(v[bt][i], inv, 12582912.f)) + (0x808080u - 0x4B400000u)) ^ 0x808080u;
        uint32_t dg[3][2];  // [digit][word]: 8 digit bytes of this lane (digit 0 = d1, the top byte)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          const uint32_t b = 2u - j;  // byte of z holding digit j
          const uint32_t sel = b | ((4u + b) << 4);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t lo = __byte_perm(z[4 * h], z[4 * h + 1], sel);
            const uint32_t hi = __byte_perm(z[4 * h + 2], z[4 * h + 3], sel);
            dg[j][h] = __byte_perm(lo, hi, 0x5410u);
          }
        }
        float sum = 0.f;
        int dsum[3] = {0, 0, 0};
        if (QT == kQ4_K) {
#pragma unroll
          for (int i = 0; i < 8; ++i) sum += v[bt][i];
          sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
          sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
        } else {
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            dsum[j] = __dp4a(static_cast<int>(dg[j][0]), 0x01010101, __dp4a(static_cast<int>(dg[j][1]), 0x01010101, 0));
            dsum[j] += __shfl_xor_sync(0xFFFFFFFFu, dsum[j], 1);
            dsum[j] += __shfl_xor_sync(0xFFFFFFFFu, dsum[j], 2);
          }
        }
        if (!valid[bt]) continue;
        const int tk = tok[bt], u = un[bt];
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          uint8_t* col = smem + a.xd_off + (3 * tk + j) * a.xd_pitch + u * kUnitK;
          if (QT == kQ4_K) {
            *reinterpret_cast<uint2*>(col + 8 * lane) = make_uint2(dg[j][0], dg[j][1]);
          } else {
            // lane covers elements 8(l&3)..+7 of block l>>2: two runs of 4
            const int e0 = 8 * (lane & 3);
            uint8_t* blk = col + 32 * (lane >> 2);
            *reinterpret_cast<uint32_t*>(blk + q40_pos(e0)) = dg[j][0];
            *reinterpret_cast<uint32_t*>(blk + q40_pos(e0 + 4)) = dg[j][1];
          }
        }
        if (lane < 3) {
          const float radix = lane == 0 ? 65536.f : lane == 1 ? 256.f : 1.f;
          reinterpret_cast<float*>(smem + a.xf_off)[u * kDCols + 3 * tk + lane] = s * radix;
        }
        if ((lane & 3) == 0) {
          if (QT == kQ4_K) {
            // sums of x per 32-weight sub-block as bf16 hi + lo: coef column 2 tok (hi)
            // and 2 tok + 1 (lo), slot j = sub-block
            const int j = lane >> 2;
            const __nv_bfloat16 hi = __float2bfloat16_rn(sum);
            const __nv_bfloat16 lo = __float2bfloat16_rn(sum - __bfloat162float(hi));
            __nv_bfloat16* e = reinterpret_cast<__nv_bfloat16*>(smem + a.xs_off) + (u * kCCols + 2 * tk) * 8 + j;
            e[0] = hi;
            e[8] = lo;
          } else {
            // C operand of each block's MMA: -8 * (sum of the block's digits) per digit column
            int* cw = reinterpret_cast<int*>(smem + a.xs_off) + (u * 8 + (lane >> 2)) * kDCols + 3 * tk;
            cw[0] = -8 * dsum[0];
            cw[1] = -8 * dsum[1];
            cw[2] = -8 * dsum[2];
          }
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"r"((W + 1) * 32) : "memory");  // x staged (all but the producer)

    if (warp == W + 1) {
      // ---------------- epilogue ----------------
      float gv[8];  // SwiGLU: this lane's gate sums of the current pair (one per token pass)
      float pv[8];  // all-reduce: this lane's partials of the current row block
      uint32_t tp_gen = 0;  // all-reduce: this call's generation (this CTA's counter + 1)
#pragma unroll
      for (int i = 0; i < 8; ++i) gv[i] = 0.f;
      for (int64_t blk = 0; blk < my_blocks; ++blk) {
        const int b = static_cast<int>(blk & 1);
        if (!mbar_wait(&rfull[b], static_cast<uint32_t>((blk >> 1) & 1))) break;
        const int64_t rb = block_of<EXT>(a, cid, ncl, blk);
        const float* rbuf = red + b * (W * a.red_stride);
        int64_t r0;
        const Seg& sg = block_rows<EXT>(a, rb, r0);
        float* xslot = reinterpret_cast<float*>(smem + a.xchg_off) + b * (8 * kRows);
        if (rank == 1 && blk >= 2 && !mbar_wait_cluster(&xempty[b], static_cast<uint32_t>(((blk >> 1) - 1) & 1))) break;
        if (rank == 0 && a.ksplit == 2 && !mbar_wait_cluster(&xfull[b], static_cast<uint32_t>((blk >> 1) & 1))) break;
        // lane = (row, half): rows on consecutive lanes read consecutive words of
        // the column-major partials (no bank conflicts); each half sums W/2 warps
        auto out_pass = [&](int it) {  // outputs of token `it` (lane = row, half)
          const int i = lane + 32 * it;
          const int row = i & 15, half = (i >> 4) & 1, tok = i >> 5;
          float v = 0.f;
#pragma unroll
          for (int w = half * (W / 2); w < (half + 1) * (W / 2); ++w) {
            const float* rw = rbuf + w * a.red_stride;
            v += rw[(3 * tok) * kRows + row] + rw[(3 * tok + 1) * kRows + row] + rw[(3 * tok + 2) * kRows + row];
            if (QT == kQ4_K) v -= rw[kRows * kDCols + tok * kRows + row];
          }
          v += __shfl_xor_sync(0xFFFFFFFFu, v, 16);
          const int64_t n_idx = r0 + phys_row(row, a.rg);
          if (rank == 1) {
            // this CTA's K half goes to rank 0, which adds it and stores y
            if (half == 0) st_cluster_f32(cluster_addr(xslot + tok * kRows + row, 0), v);
            return;
          }
          if (a.ksplit == 2) v += xslot[tok * kRows + row];
          if constexpr (EXT) {
            if (a.swiglu) {
              if ((blk & 1) == 0) {
                gv[it] = v;  // gate: kept until the up rows of the pair
                return;
              }
              const float g = gv[it];
              v = g / (1.f + __expf(-g)) * v;  // silu(gate) * up
            }
            if (a.tp_world > 1) {
              pv[it] = v;  // joined with the other GPUs' partials below
              return;
            }
          }
          const Seg& so = EXT && a.swiglu ? a.seg[0] : sg;
          if (half == 0 && n_idx < so.n) {
            if (EXT && a.resid) v += load_y_rt(a.resid, a.ytype, tok * a.ldr + n_idx);
            store_y_rt(so.y, a.ytype, tok * so.ldy + n_idx, v);
          }
        };
        if constexpr (EXT) {
#pragma unroll
          for (int it = 0; it < 8; ++it) {  // registers gv / pv need static indices
            if (it >= a.m) break;
            out_pass(it);
          }
        } else {
          for (int it = 0; it < a.m; ++it) out_pass(it);
        }
        if (EXT && a.tp_world > 1 && rank == 0) {
          // this GPU's partials of the row block into every GPU's slot [gen & 1][tp_rank],
          // each value with the call's generation in the same 8-byte word (the receiver
          // polls the words themselves: no fence, no flag)
          if (blk == 0 && lane == 0)
            tp_gen = *reinterpret_cast<volatile uint32_t*>(reinterpret_cast<uint32_t*>(a.peer[a.tp_rank]) + cid) + 1u;
          tp_gen = __shfl_sync(0xFFFFFFFFu, tp_gen, 0);
          const uint64_t tag = static_cast<uint64_t>(tp_gen) << 32;
          const int64_t par = tp_gen & 1u;
          const int64_t nb = a.seg[0].n;
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            if (it >= a.m) break;
            const int i = lane + 32 * it;
            const int row = i & 15, half = (i >> 4) & 1, tok = i >> 5;
            const int64_t n_idx = r0 + phys_row(row, a.rg);
            if (half == 0 && n_idx < nb) {
              const int64_t off = ((par * a.tp_world + a.tp_rank) * a.m_max + tok) * nb + n_idx;
              const uint64_t w = tag | __float_as_uint(pv[it]);
              for (int p = 0; p < a.tp_world; ++p)
                st_relaxed_sys_u64(reinterpret_cast<uint64_t*>(a.peer[p] + kTpHdr) + off, w);
            }
          }
        }
        if (rank == 1) {
          asm volatile("fence.acq_rel.cluster;" ::: "memory");
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(cluster_addr(&xfull[b], 0));
        } else if (a.ksplit == 2) {
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(cluster_addr(&xempty[b], 1));
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rempty[b]);
      }
      if (EXT && a.tp_world > 1 && rank == 0 && my_blocks > 0) {
        // the other GPUs' partials of the same row blocks (same CTA index: the row-block
        // schedule is the same on every GPU) arrive as tagged words in this GPU's buffer:
        // poll each until it carries this call's generation (bounded), then the sums in
        // rank order -- the same bits on every GPU
        const int64_t par = tp_gen & 1u;
        const int64_t nb = a.seg[0].n;
        const uint64_t* mine = reinterpret_cast<const uint64_t*>(a.peer[a.tp_rank] + kTpHdr);
        const uint32_t lim = g_wait_limit;
        bool ok2 = true;
        for (int64_t blk = 0; blk < my_blocks && ok2; ++blk) {
          int64_t r0;
          block_rows<EXT>(a, block_of<EXT>(a, cid, ncl, blk), r0);
          for (int i = lane; i < kRows * a.m && ok2; i += 32) {
            const int row = i & 15, tok = i >> 4;
            const int64_t n_idx = r0 + phys_row(row, a.rg);
            if (n_idx < nb) {
              float v = 0.f;
              for (int p = 0; p < a.tp_world && ok2; ++p) {
                const uint64_t* src = mine + ((par * a.tp_world + p) * a.m_max + tok) * nb + n_idx;
                uint64_t w = 0;
                ok2 = false;
                for (uint32_t q = 0; q < lim; ++q) {
                  w = ld_relaxed_sys_u64(src);
                  if (static_cast<uint32_t>(w >> 32) == tp_gen) {
                    ok2 = true;
                    break;
                  }
                  if (q > 64) __nanosleep(32);
                }
                v += __uint_as_float(static_cast<uint32_t>(w));
              }
              if (!ok2) break;
              if (a.resid) v += load_y_rt(a.resid, a.ytype, tok * a.ldr + n_idx);
              store_y_rt(a.seg[0].y, a.ytype, tok * a.seg[0].ldy + n_idx, v);
            }
          }
          ok2 = __all_sync(0xFFFFFFFFu, ok2);
        }
        if (!ok2 && lane == 0) atomicOr(&g_device_error, kErrWaitTimeout);
        __syncwarp();
        if (lane == 0) reinterpret_cast<uint32_t*>(a.peer[a.tp_rank])[cid] = tp_gen;  // this CTA's call done
      }
    } else {
      // ---------------- compute ----------------
      const int dcols = 3 * a.m, ccols = 2 * a.m;
      uint32_t xcol[NCG];
#pragma unroll
      for (int cg = 0; cg < NCG; ++cg) {
        const int col = cg * 8 + g < dcols ? cg * 8 + g : 0;  // unused B columns read column 0
        xcol[cg] = a.xd_off + col * a.xd_pitch + 8u * t;
      }
      const int ccol = g < ccols ? g : 0;
      const uint32_t roff_g = row_off(phys_row(g, a.rg), a), roff_g8 = row_off(phys_row(g + 8, a.rg), a);
      float ft[NCG][4], ft2[NCG][4];
      float cmin[2 * NCC], cmin2[2 * NCC];
#pragma unroll
      for (int cg = 0; cg < NCG; ++cg)
#pragma unroll
        for (int i = 0; i < 4; ++i) ft[cg][i] = ft2[cg][i] = 0.f;
#pragma unroll
      for (int i = 0; i < 2 * NCC; ++i) cmin[i] = cmin2[i] = 0.f;
      int64_t p = 0;
      bool ok = true;
      for (int64_t blk = 0; blk < my_blocks && ok; ++blk) {
        for (int ch = 0; ch < a.nchunks; ++ch, ++p) {
          const int s = static_cast<int>(p % a.stages);
          if (!mbar_wait(&full[s], static_cast<uint32_t>((p / a.stages) & 1))) {
            ok = false;
            break;
          }
          const int nu = min(a.chunk_units, units - ch * a.chunk_units);
          const uint32_t sbase = static_cast<uint32_t>(s * a.stage_bytes);
          auto ctx = [&](int uu) {
            const int ku = ch * a.chunk_units + uu;  // unit index along K
            Ctx c;
            c.smem = smem;
            c.rg = sbase + roff_g + uu * a.unit_bytes;
            c.rg8 = sbase + roff_g8 + uu * a.unit_bytes;
#pragma unroll
            for (int cg = 0; cg < NCG; ++cg) c.xo[cg] = xcol[cg] + ku * kUnitK;
            c.xf = a.xf_off + (ku * kDCols + 2 * t) * 4u;
            if (QT == kQ4_K) c.xs = a.xs_off + ((ku * kCCols + ccol) * 8 + 2 * t) * 2u;
            else c.xs = a.xs_off + ((ku * 8) * kDCols + 2 * t) * 4u;
            c.t = t;
            return c;
          };
          int uu = warp;
          // two units at a time, with separate accumulators
          for (; W <= 8 && uu + W < nu; uu += 2 * W) {
            const Ctx c0 = ctx(uu), c1 = ctx(uu + W);
            if (QT == kQ4_K) {
              unit_q4k<NCG, NCC>(c0, ft, cmin);
              unit_q4k<NCG, NCC>(c1, ft2, cmin2);
            } else {
              unit_q40<NCG>(c0, ft);
              unit_q40<NCG>(c1, ft2);
            }
          }
          for (; uu < nu; uu += W) {
            if (QT == kQ4_K) unit_q4k<NCG, NCC>(ctx(uu), ft, cmin);
            else unit_q40<NCG>(ctx(uu), ft);
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (!ok) break;
        const int b = static_cast<int>(blk & 1);
        if (blk >= kRedBufs && !mbar_wait(&rempty[b], static_cast<uint32_t>(((blk >> 1) - 1) & 1))) break;
        float* rw = red + b * (W * a.red_stride) + warp * a.red_stride;
#pragma unroll
        for (int cg = 0; cg < NCG; ++cg) {  // column-major [col][16 rows]
          const int c0 = cg * 8 + 2 * t;
          rw[c0 * kRows + g] = ft[cg][0] + ft2[cg][0];
          rw[(c0 + 1) * kRows + g] = ft[cg][1] + ft2[cg][1];
          rw[c0 * kRows + g + 8] = ft[cg][2] + ft2[cg][2];
          rw[(c0 + 1) * kRows + g + 8] = ft[cg][3] + ft2[cg][3];
#pragma unroll
          for (int i = 0; i < 4; ++i) ft[cg][i] = ft2[cg][i] = 0.f;
        }
        if (QT == kQ4_K) {
          float* rc = rw + kRows * kDCols;  // [8 tokens][16 rows]
#pragma unroll
          for (int cc = 0; cc < NCC; ++cc) {
            rc[(4 * cc + t) * kRows + g] = cmin[2 * cc] + cmin2[2 * cc];
            rc[(4 * cc + t) * kRows + g + 8] = cmin[2 * cc + 1] + cmin2[2 * cc + 1];
          }
#pragma unroll
          for (int i = 0; i < 2 * NCC; ++i) cmin[i] = cmin2[i] = 0.f;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rfull[b]);
      }
    }
  }
  __syncthreads();
  // neither CTA of a cluster leaves while the other may still touch its shared memory
  if (a.ksplit == 2) cluster_sync_all();
  // a bounded wait may have given up: no copy of this CTA may still be in flight at exit
  if (warp == W && lane == 0) {
    for (int64_t q = total_pieces - a.stages; q < total_pieces; ++q)
      if (q >= 0) mbar_wait(&full[q % a.stages], static_cast<uint32_t>((q / a.stages) & 1));
  }
}

int ncg_of(int m) { return (3 * m + 7) / 8; }

bool plan_i8(int qt, int64_t k, int m, int smem_budget, int W, int ksplit, I8Args& a) {
  if (qt != kQ4_K && qt != kQ4_0) return false;
  if (k % kUnitK || m < 1 || m > 8 || k > (1 << 20)) return false;
  if (k % (ksplit * kUnitK)) return false;
  a.ksplit = ksplit;
  a.unit_bytes = 144;  // one Q4_K superblock = 8 Q4_0 blocks = 144 bytes
  const int ncg = ncg_of(m), ncc = ncg == 1 ? 1 : 2;
  const int units = static_cast<int>(k / kUnitK) / ksplit;  // per CTA
  a.xd_pitch = units * kUnitK + 32;
  const int xd_bytes = 3 * m * a.xd_pitch;
  const int xf_bytes = units * 8 * ncg * 4;
  const int xs_bytes = qt == kQ4_K ? units * 8 * ncc * 8 * 2 : units * 8 * 8 * ncg * 4;
  // + 4 floats: the two halves of the epilogue warp (4 or 8 warps apart) hit different banks
  a.red_stride = kRows * 8 * ncg + (qt == kQ4_K ? kRows * 8 : 0) + 4;
  const int red_bytes = kRedBufs * W * a.red_stride * 4;
  const int xchg_bytes = ksplit == 2 ? 2 * 8 * kRows * 4 : 0;
  const int fixed = xd_bytes + xf_bytes + xs_bytes + red_bytes + xchg_bytes + 20 * 8 + 64;
  // Pieces: 16 rows x a chunk of up to 32 units (4608 bytes a row), else 16 units;
  // copies of >= 4 KB where possible (short bulk copies are request-bound).
  int stages = 0;
  for (int cu_max : {32, 16}) {
    a.chunk_units = std::min(units, cu_max);
    a.nchunks = (units + a.chunk_units - 1) / a.chunk_units;
    a.chunk_bytes = a.chunk_units * a.unit_bytes;
    a.rg = 1;
    if (a.nchunks == 1 && ksplit == 1)  // rows contiguous only when a chunk is the whole row
      while (a.rg < 8 && 2 * a.rg * a.chunk_bytes <= kCopyBytes) a.rg *= 2;
    a.group_pitch = (a.rg * a.chunk_bytes + 127) / 128 * 128 + 32;  // 32 mod 128: conflict-free reads
    a.stage_bytes = (kRows / a.rg) * a.group_pitch;
    stages = std::min(6, (smem_budget - fixed) / a.stage_bytes);
    if (stages >= 2) break;
  }
  if (stages < 2) return false;
  a.stages = stages;
  a.xd_off = static_cast<uint32_t>(stages * a.stage_bytes);
  a.xf_off = a.xd_off + (xd_bytes + 15) / 16 * 16;
  a.xs_off = a.xf_off + xf_bytes;
  a.red_off = a.xs_off + (xs_bytes + 15) / 16 * 16;
  a.xchg_off = a.red_off + red_bytes;
  a.bar_off = (a.xchg_off + xchg_bytes + 7) / 8 * 8;
  return true;
}

std::mutex g_attr_mu;
std::set<std::pair<const void*, int>> g_attr_done;

template <int QT, int NCG, int W, bool EXT, int MINB>
cudaError_t launch_t(I8Args& a, int dev, int sms, int smem_optin, cudaStream_t st) {
  constexpr int NCC = NCG == 1 ? 1 : 2;
  auto fn = gemv_i8_kernel<QT, NCG, NCC, W, EXT, MINB>;
  const int smem = static_cast<int>(a.bar_off + 8 * (2 * a.stages + 2 * kRedBufs + 4));
  {
    std::lock_guard<std::mutex> lk(g_attr_mu);
    if (!g_attr_done.count({reinterpret_cast<const void*>(fn), dev})) {
      cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin);
      if (e != cudaSuccess) return e;
      g_attr_done.insert({reinterpret_cast<const void*>(fn), dev});
    }
  }
  cudaLaunchConfig_t cfg = {};
  // sms = CTA slots; with the K split a cluster of 2 takes two of them
  cfg.gridDim = dim3(static_cast<unsigned>(a.ksplit * std::min<int64_t>(a.nrowblocks, sms / a.ksplit)));
  cfg.blockDim = dim3((W + 2) * 32);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = a.ksplit;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = a.ksplit == 2 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, fn, a);
}

template <int QT, int W, int MINB>
cudaError_t launch_q(I8Args& a, int dev, int sms, int smem_optin, cudaStream_t st) {
  const bool ext = a.swiglu || a.tp_world > 1 || a.resid;
  switch (ncg_of(a.m)) {
    case 1: return ext ? launch_t<QT, 1, W, true, MINB>(a, dev, sms, smem_optin, st) : launch_t<QT, 1, W, false, MINB>(a, dev, sms, smem_optin, st);
    case 2: return ext ? launch_t<QT, 2, W, true, MINB>(a, dev, sms, smem_optin, st) : launch_t<QT, 2, W, false, MINB>(a, dev, sms, smem_optin, st);
    default: return ext ? launch_t<QT, 3, W, true, MINB>(a, dev, sms, smem_optin, st) : launch_t<QT, 3, W, false, MINB>(a, dev, sms, smem_optin, st);
  }
}

// CTA shape: 4 compute warps in <= 113 KB of shared memory, two CTAs per SM
// (the next launch's CTAs become resident, and start streaming their weights,
// as soon as any CTA of the previous one exits), when the activations and two
// ring stages fit; else 8 compute warps, one CTA per SM. GGUFMM_GEMV_WARPS=8
// forces the one-CTA shape (tuning).
int forced_warps() {
  static const int w = [] {
    const char* e = std::getenv("GGUFMM_GEMV_WARPS");
    const int v = e ? std::atoi(e) : 0;
    return v == 8 ? v : 0;
  }();
  return w;
}
// GGUFMM_GEMV_KSPLIT=1: split K over the two CTAs of a cluster whenever the 4-warp
// shape does not fit; =2: only when the row blocks are too few to give every SM two
// of them. Off by default: on the 4096 x 14336 down projection the one-CTA 8-warp
// shape measured 13.4 us per launch against 14.4 us for the split.
int ksplit_mode() {
  static const int v = [] {
    const char* e = std::getenv("GGUFMM_GEMV_KSPLIT");
    return e && (e[0] == '1' || e[0] == '2') ? e[0] - '0' : 0;
  }();
  return v;
}
// Shapes: 4 = 4 compute warps, two CTAs per SM; 82 = 8 compute warps, two CTAs per SM
// (registers capped at 96); 8 = 8 compute warps, one CTA per SM.
int smem_of(int W, int optin) { return std::min(optin, W == 4 || W == 82 ? 113 * 1024 : 227 * 1024); }
// GGUFMM_GEMV_SHAPE=8x2 selects the 8-warp two-CTA shape where it fits (tuning).
bool shape_8x2() {
  static const bool on = [] {
    const char* e = std::getenv("GGUFMM_GEMV_SHAPE");
    return e && e[0] == '8' && e[1] == 'x';
  }();
  return on;
}
// rowblocks: 16-row blocks of the launch (0 when only asking whether a plan exists).
int pick_warps(int qt, int64_t k, int m, int optin, I8Args& a, int64_t rowblocks = 0, int sms = 0) {
  const int f = forced_warps();
  if (f) return plan_i8(qt, k, m, smem_of(f, optin), f, 1, a) ? f : 0;
  if (shape_8x2() && plan_i8(qt, k, m, smem_of(82, optin), 8, 1, a)) return 82;
  if (plan_i8(qt, k, m, smem_of(4, optin), 4, 1, a)) return 4;
  // Too large for one half-SM CTA: one 8-warp CTA per SM, or -- where even that
  // does not fit (the activations of M = 8 at K = 14336), or where asked for --
  // K split over the two CTAs of a cluster.
  const bool few_rows = rowblocks > 0 && rowblocks < 2 * static_cast<int64_t>(sms);
  const bool prefer_split = ksplit_mode() == 1 || (ksplit_mode() == 2 && few_rows);
  const bool w8 = plan_i8(qt, k, m, smem_of(8, optin), 8, 1, a);
  if ((prefer_split || !w8) && plan_i8(qt, k, m, smem_of(4, optin), 4, 2, a)) return 4;
  return w8 && plan_i8(qt, k, m, smem_of(8, optin), 8, 1, a) ? 8 : 0;
}

// GGUFMM_GEMV_IMPL=f16 turns this path off (the fp16 tensor-core GEMV then runs).
bool i8_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GGUFMM_GEMV_IMPL");
    return !(e && e[0] == 'f');
  }();
  return on;
}

}  // namespace

struct DevInfo {
  int sms = 0;
  int smem_optin = 0;
};
DevInfo device_info(int dev);  // capi.cu

bool gemv_i8_supported(int qtype, int64_t k, int m) {
  if (!i8_enabled()) return false;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  const DevInfo di = device_info(dev);
  I8Args a{};
  return pick_warps(qtype, k, m, di.smem_optin, a) != 0;
}

// nseg weights of one qtype and K (16-byte aligned bases, row bytes a multiple
// of 16) against the same activations, one launch.
// swiglu: nseg = 2 (gate, up) of equal N; y[0] receives silu(x Wg^T) * (x Wu^T).
// tp (optional): all-reduce y over tp->world GPUs through their exchange buffers.
// resid (optional, nseg = 1, no swiglu): y = x W^T + resid, resid in y's dtype with row stride ldr
// (it may be y itself for an in-place residual add).
struct GemvTp {
  int world, rank;
  uint32_t epoch;
  int64_t m_max;
  const void* const* bufs;
};
size_t gemv_tp_buffer_bytes(int64_t n, int64_t m_max, int world) {
  return kTpHdr + (static_cast<size_t>(2) * world * m_max * n * 8 + 255) / 256 * 256;
}

cudaError_t launch_gemv_i8_grouped(int nseg, const void* const* q, const int64_t* n, int qtype, int64_t k,
                                   const void* x, int xtype, int64_t m, int64_t ldx, void* const* y, int ytype,
                                   const int64_t* ldy, int64_t row_bytes, cudaStream_t st, int swiglu,
                                   const GemvTp* tp, const void* resid, int64_t ldr) {
  if (nseg < 1 || nseg > kMaxSegs) return cudaErrorInvalidValue;
  if (resid && (nseg != 1 || swiglu)) return cudaErrorInvalidValue;
  if (swiglu && (nseg != 2 || n[0] != n[1])) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const DevInfo di = device_info(dev);
  I8Args a{};
  int64_t nrb = 0;
  for (int i = 0; i < nseg; ++i) nrb += (n[i] + kRows - 1) / kRows;
  const int shape = pick_warps(qtype, k, static_cast<int>(m), di.smem_optin, a, nrb, di.sms);
  if (!shape) return cudaErrorInvalidValue;
  const int optin = smem_of(shape, di.smem_optin);
  a.nseg = nseg;
  int64_t rb = 0;
  for (int i = 0; i < nseg; ++i) {
    a.seg[i].q = static_cast<const uint8_t*>(q[i]);
    a.seg[i].y = y[i];
    a.seg[i].n = n[i];
    a.seg[i].ldy = ldy[i];
    a.seg[i].rb0 = rb;
    rb += (n[i] + kRows - 1) / kRows;
  }
  a.nrowblocks = rb;
  a.swiglu = swiglu;
  a.resid = resid;
  a.ldr = ldr;
  a.tp_world = 1;
  if (tp && tp->world > 1) {
    if (nseg != 1 || swiglu || tp->world > 8 || m > tp->m_max) return cudaErrorInvalidValue;
    a.tp_world = tp->world;
    a.tp_rank = tp->rank;
    a.epoch = tp->epoch;
    a.m_max = tp->m_max;
    a.tp_nrb = rb;
    a.tp_flag_off = 0;
    for (int i = 0; i < tp->world; ++i) a.peer[i] = reinterpret_cast<uint64_t>(tp->bufs[i]);
  }
  a.k = static_cast<int>(k);
  a.row_bytes = row_bytes;
  a.x = x;
  a.xtype = xtype;
  a.ldx = ldx;
  a.m = static_cast<int>(m);
  a.ytype = ytype;
  if (shape == 4) return qtype == kQ4_K ? launch_q<kQ4_K, 4, 2>(a, dev, 2 * di.sms, optin, st)
                                        : launch_q<kQ4_0, 4, 2>(a, dev, 2 * di.sms, optin, st);
  if (shape == 82) return qtype == kQ4_K ? launch_q<kQ4_K, 8, 2>(a, dev, 2 * di.sms, optin, st)
                                         : launch_q<kQ4_0, 8, 2>(a, dev, 2 * di.sms, optin, st);
  return qtype == kQ4_K ? launch_q<kQ4_K, 8, 1>(a, dev, di.sms, optin, st)
                        : launch_q<kQ4_0, 8, 1>(a, dev, di.sms, optin, st);
}

cudaError_t gemv_i8_device_error(int* v, int clear, cudaStream_t st) { return tu_device_error(v, clear, st); }
cudaError_t gemv_i8_set_wait_limit(uint32_t polls) { return tu_set_wait_limit(polls); }

}  // namespace ggufmm
