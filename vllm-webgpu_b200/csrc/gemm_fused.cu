// gemm_fused.cu -- Q4_K GEMM on the sm_100a tensor cores with the dequantization
// fused into the pipeline: Y[m, n] = sum_k X[m, k] W[n, k] (batched decode and short prefill).
//
// The two-pass GEMM (dequantize the whole weight to fp16 in scratch, then a
// tcgen05 GEMM) moves 4.5 bytes per weight through HBM (0.56 read, 2 written,
// 2 read again). Here each CTA streams the packed GGUF bytes of its 128 weight
// rows once (0.56 B per weight) and turns them into the fp16 MMA operand in
// tensor memory, next to the tensor cores.
//
// CTA = 14 warps, one 128 (weight rows, MMA M) x BN (tokens, MMA N) tile:
//   warp 0       TMA producer: per 128-weight k-block, the rows' 16-byte Q4_K
//                headers (d, dmin, 6-bit scales) and 64 bytes of nibbles (2-D
//                uint8 tensor maps, 64-byte swizzle for the nibbles), and the
//                activation tile (fp16, 128-byte swizzle); one mbarrier
//                transaction count per stage.
//   warps 6..13  dequantizers: thread (row r, half q) decodes the 64 weights of
//                one nibble chunk to fp32 exactly as gguf-py does
//                ((d*sc)*q - dmin*m; the product is exact, so one fma), rounds
//                once to fp16 and stores them with tcgen05.st into TMEM lane r,
//                where tcgen05.mma reads its A operand.
//   warp 1       allocates TMEM and issues tcgen05.mma (kind::f16, A in TMEM,
//                B in shared memory, M=128, N=BN, K=16) from one elected lane;
//                each stage is committed back to the producer, the last one to
//                the epilogue.
//   warps 2..5   epilogue: tcgen05.ld of the fp32 accumulator, transposed
//                stores of Y.
// Operand precision is that of the two-pass GEMM: the exact fp32 dequantized
// weight rounded once to fp16, activations in fp16, fp32 accumulation.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <utility>

#include "tcgen05.cuh"

namespace ggufmm {

constexpr int kFKB = 128;      // weights per k-block (half a Q4_K superblock)
constexpr int kFusedThreads = 14 * 32;

// Two fp32 lanes in one instruction (sm_100 packed f32x2): (m - 2^23) * ds + nd per
// lane, each lane rounded exactly as the scalar sub and fma would round it.
__device__ __forceinline__ uint32_t dequant_pair_f16(uint32_t m0, uint32_t m1, uint64_t ds2, uint64_t nd2) {
  uint64_t v, t;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(m0), "r"(m1));
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(t) : "l"(v), "l"(0x4B0000004B000000ull));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(v) : "l"(ds2), "l"(t), "l"(nd2));
  float f0, f1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(f0), "=f"(f1) : "l"(v));
  __half2 h2 = __floats2half2_rn(f0, f1);
  return *reinterpret_cast<uint32_t*>(&h2);
}
__device__ __forceinline__ uint64_t splat2(float f) {
  return (static_cast<uint64_t>(__float_as_uint(f)) << 32) | __float_as_uint(f);
}

// Exact float of a small non-negative integer (< 2^22).
__device__ __forceinline__ float small_uint_to_float(uint32_t v) {
  return __fsub_rn(__uint_as_float(0x4B000000u | v), 8388608.f);
}

// Up to kMaxFusedSegs weights of one K that read the same activations (q/k/v,
// gate/up): segment s owns row tiles [tile0[s], tile0[s + 1]) of the grid's y
// dimension and global rows [row0[s], row0[s + 1]) of the K split's partials.
constexpr int kMaxFusedSegs = 4;
struct FusedSegs {
  CUtensorMap hdr[kMaxFusedSegs];  // 16-byte Q4_K headers, box 16 B x 128 rows
  CUtensorMap qs[kMaxFusedSegs];   // nibbles, box 64 B x 128 rows
  void* y[kMaxFusedSegs];
  int64_t ldy[kMaxFusedSegs];
  int n[kMaxFusedSegs];
  int tile0[kMaxFusedSegs + 1];
  int row0[kMaxFusedSegs + 1];
  int nseg;
  int64_t row_bytes;
};

// ---- the same GEMM with the dequantized operand in tensor memory ----------------
// tcgen05.mma can read its A operand from TMEM instead of shared memory. Here the
// dequantizer threads (one weight row = one TMEM lane each) write the fp16 weights
// of a k-block straight into TMEM with tcgen05.st, and the MMA reads them there:
// shared memory then carries only the TMA traffic (headers, nibbles, activations)
// and the nibble reads -- about 1.1 bytes per weight instead of 5.1 with the
// operand staged through shared memory and read back by the tensor core.
// TMEM columns: [0, BN) the fp32 accumulator, [128 + 64 s, 128 + 64 (s + 1)) the
// 128 x 128 fp16 A operand of ring stage s (row = lane, two k per 32-bit column).
template <int BN, int OCC = 1>
struct FusedTmemSmem {
  static constexpr uint32_t kB = BN * kFKB * 2;      // activation tile, 2 SW128 atoms
  static constexpr uint32_t kHdr = kTileW * 16;
  static constexpr uint32_t kQs = kTileW * 64;       // 64-byte swizzled nibble rows
  static constexpr uint32_t kStage = kB + kHdr + kQs;
  // OCC = 2: two CTAs per SM, each with 256 TMEM columns (accumulator + 3 A stages)
  static constexpr int kMaxStages = OCC == 2 ? 3 : 6;
  static constexpr int kStages = (224 * 1024 / OCC) / kStage < kMaxStages ? (224 * 1024 / OCC) / kStage : kMaxStages;
  static constexpr uint32_t kBarOff = kStages * kStage;
  static constexpr uint32_t kTotal = kBarOff + (4 * kStages + 1) * 8 + 16 + 1024;
  static constexpr uint32_t kAcol = OCC == 2 ? 64 : (BN > 128 ? BN : 128);  // first A column
  static constexpr uint32_t kCols = OCC == 2 ? 256 : 512;
  static_assert(OCC == 1 || BN <= 64, "two CTAs per SM hold at most 64 accumulator columns");
  static_assert(kAcol + 64 * kStages <= kCols, "accumulator and operand stages exceed the TMEM allocation");
};

__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(v[0]), "r"(v[1]),
               "r"(v[2]), "r"(v[3])
               : "memory");
}

template <int BN, int OCC>
__global__ void __launch_bounds__(kFusedThreads, OCC)
    gemm_fused_q4k_tmem_kernel(const __grid_constant__ FusedSegs sg, const __grid_constant__ CUtensorMap tm_x,
                               int ytype, int m, int k, float* __restrict__ part, int kb_per) {
  using L = FusedTmemSmem<BN, OCC>;
  constexpr int S = L::kStages;
  constexpr uint32_t kCols = L::kCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // full[s]: the stage's weight blocks landed (dequantizers); xfull[s]: its activation
  // tile landed (MMA) -- separate so the dequantizers can start on the weights, which
  // are streamed before the previous kernel has finished, without waiting for x
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* afull = full + S;
  uint64_t* empty = afull + S;
  uint64_t* xfull = empty + S;
  uint64_t* accum = xfull + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int seg = 0;
  while (seg + 1 < sg.nseg && static_cast<int>(blockIdx.y) >= sg.tile0[seg + 1]) ++seg;
  const int m0 = blockIdx.x * BN, n0 = (static_cast<int>(blockIdx.y) - sg.tile0[seg]) * kTileW;
  const int n = sg.n[seg];
  const int kb0 = blockIdx.z * kb_per;
  const int nkb = min(k / kFKB - kb0, kb_per);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&afull[s], 8);
      mbar_init(&empty[s], 1);
      mbar_init(&xfull[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_d = *tmem_slot;

  pdl_trigger();
  if (warp == 0) {
    if (lane == 0) {
      // the weights are read-only: the first stages' blocks stream in before the
      // previous kernel (which writes x and reads y / the partials) has finished
      auto load_w = [&](int i) {
        const int s = i % S, kb = kb0 + i;
        uint8_t* st = smem + s * L::kStage;
        const int sb = kb >> 1, h = kb & 1;
        mbar_arrive_expect_tx(&full[s], L::kHdr + L::kQs);
        tma_load_2d(st + L::kB, &sg.hdr[seg], 144 * sb, n0, &full[s]);
        tma_load_2d(st + L::kB + L::kHdr, &sg.qs[seg], 144 * sb + 16 + 64 * h, n0, &full[s]);
      };
      const int pre = min(S, nkb);
      for (int i = 0; i < pre; ++i) load_w(i);
      pdl_wait();
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S, kb = kb0 + i;
        if (i >= pre) {
          if (!mbar_wait(&empty[s], ((i / S) & 1) ^ 1)) break;
          load_w(i);
        }
        uint8_t* st = smem + s * L::kStage;
        mbar_arrive_expect_tx(&xfull[s], L::kB);
        tma_load_2d(st, &tm_x, kb * kFKB, m0, &xfull[s]);
        tma_load_2d(st + BN * 128, &tm_x, kb * kFKB + 64, m0, &xfull[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16<BN>();
      for (int i = 0; i < nkb; ++i) {
        const int s = i % S;
        const uint32_t par = (i / S) & 1;
        if (!mbar_wait(&xfull[s], par) || !mbar_wait(&afull[s], par)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t b_addr = smem_u32(smem + s * L::kStage);
        const uint32_t a_col = tmem_d + L::kAcol + 64u * s;
#pragma unroll
        for (int atom = 0; atom < 2; ++atom) {
          const uint64_t bdesc = umma_smem_desc(b_addr + atom * (BN * 128));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_ts(tmem_d, a_col + 32 * atom + 8 * kk, bdesc + 2 * kk, idesc,
                        (i > 0 || atom > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);
    }
  } else if (warp < 6) {
    const int quad = warp & 3;
    pdl_wait();  // y / the partials may still be read by the previous kernel
    const bool ok = mbar_wait(accum, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok) {
      const int nrow = n0 + quad * 32 + lane;
      void* const y = sg.y[seg];
      const int64_t ldy = sg.ldy[seg];
      const int64_t ntot = sg.row0[sg.nseg], grow = sg.row0[seg] + nrow;
      const uint32_t tbase = tmem_d + (static_cast<uint32_t>(quad * 32) << 16);
      constexpr int kEpiChunk = 32;
      if (part) {
        float* pz = part + static_cast<int64_t>(blockIdx.z) * m * ntot + grow;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += kEpiChunk) {
          uint32_t r[kEpiChunk];
#pragma unroll
          for (int h = 0; h < kEpiChunk; h += 16) tmem_ld16_async(tbase + c0 + h, r + h);
          tmem_wait_ld();
          if (nrow < n) {
#pragma unroll
            for (int j = 0; j < kEpiChunk; ++j) {
              const int mm = m0 + c0 + j;
              if (mm < m) pz[static_cast<int64_t>(mm) * ntot] = __uint_as_float(r[j]);
            }
          }
        }
      } else if (ytype == GGUFMM_BF16) {
        drain_tile<BN, GGUFMM_BF16, kEpiChunk>(tbase, y, ldy, m0, m, nrow, n);
      } else if (ytype == GGUFMM_F32) {
        drain_tile<BN, GGUFMM_F32, kEpiChunk>(tbase, y, ldy, m0, m, nrow, n);
      } else {
        drain_tile<BN, GGUFMM_F16, kEpiChunk>(tbase, y, ldy, m0, m, nrow, n);
      }
    }
  } else {
    // dequantizers: warp w owns TMEM lanes 32 (w % 4) .. + 31, so thread (row r =
    // 32 (w % 4) + lane, 64-weight half q of the k-block) writes its own lane
    const int r = ((warp & 3) << 5) | lane, q = (warp - 6) >> 2;
    const uint32_t trow = tmem_d + (static_cast<uint32_t>(warp & 3) << 21) + L::kAcol + 32u * q;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % S, kb = kb0 + i;
      if (!mbar_wait(&full[s], (i / S) & 1)) break;
      // the MMAs that last read this stage's columns completed before the producer
      // refilled the stage (empty[s] -> full[s])
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint8_t* st = smem + s * L::kStage;
      const uint4 hd = *reinterpret_cast<const uint4*>(st + L::kB + r * 16);
      const uint8_t* qrow = st + L::kB + L::kHdr + r * 64;
      const int swz = (r >> 1) & 3;  // 64-byte swizzle of the nibble rows
      const uint4 q0 = *reinterpret_cast<const uint4*>(qrow + (((2 * q) ^ swz) << 4));
      const uint4 q1 = *reinterpret_cast<const uint4*>(qrow + (((2 * q + 1) ^ swz) << 4));
      const int c = 2 * (kb & 1) + q;
      const float d = half_bits_to_float(hd.x), dmin = half_bits_to_float(hd.x >> 16);
      const uint32_t hi_sel = 0u - static_cast<uint32_t>(c >> 1);
      const uint32_t scw = ((hd.y & 0x3F3F3F3Fu) & ~hi_sel) | (((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u)) & hi_sel);
      const uint32_t mw = ((hd.z & 0x3F3F3F3Fu) & ~hi_sel) | ((((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u)) & hi_sel);
      const uint32_t sh = 16u * (c & 1);
      const float dsc_lo = __fmul_rn(d, small_uint_to_float((scw >> sh) & 0xFFu));
      const float dsc_hi = __fmul_rn(d, small_uint_to_float((scw >> (sh + 8)) & 0xFFu));
      const float ndm_lo = -__fmul_rn(dmin, small_uint_to_float((mw >> sh) & 0xFFu));
      const float ndm_hi = -__fmul_rn(dmin, small_uint_to_float((mw >> (sh + 8)) & 0xFFu));
      const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
      for (int kc = 0; kc < 8; ++kc) {  // 8 consecutive k: low nibbles of bytes 8kc.. or high of 8(kc-4)..
        const bool hi = kc >= 4;
        const int kk = hi ? kc - 4 : kc;
        const uint32_t wa = w[kk * 2], wb = w[kk * 2 + 1];
        const int shn = hi ? 4 : 0;
        const uint64_t ds2 = splat2(hi ? dsc_hi : dsc_lo), nd2 = splat2(hi ? ndm_hi : ndm_lo);
        const uint32_t na = (wa >> shn) & 0x0F0F0F0Fu, nb = (wb >> shn) & 0x0F0F0F0Fu;
        uint32_t out[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t src = e < 2 ? na : nb;
          const uint32_t b0 = (2u * e) & 3u;
          out[e] = dequant_pair_f16(__byte_perm(src, 0x4B000000u, 0x7540u | b0),
                                    __byte_perm(src, 0x4B000000u, 0x7540u | (b0 + 1)), ds2, nd2);
        }
        tmem_st4(trow + 64u * s + 4u * kc, out);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&afull[s]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kCols) : "memory");
  }
}

// ---- host side --------------------------------------------------------------
// uint8 2-D map over the GGUF bytes [rows, row_bytes], box = box_bytes x 128 rows.
static bool make_map_q(CUtensorMap* map, const void* base, int64_t rows, int64_t row_bytes, int box_bytes,
                       CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_NONE) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_bytes), static_cast<cuuint32_t>(kTileW)};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static std::mutex g_fused_attr_mu;
static std::set<std::pair<const void*, int>> g_fused_attr_done;

// y_s[mm, row] = sum over z (in order) of part[z][mm][row0[s] + row]: the K split's
// partial sums, added in a fixed order so the result does not depend on CTA timing.
struct ReduceSegs {
  void* y[kMaxFusedSegs];
  int64_t ldy[kMaxFusedSegs];
  int row0[kMaxFusedSegs + 1];
  int nseg;
};
__global__ void fused_splitk_reduce_kernel(const float* __restrict__ part, int ks, int m, ReduceSegs rs, int ytype) {
  pdl_trigger();
  pdl_wait();
  const int ntot = rs.row0[rs.nseg];
  const int64_t total = static_cast<int64_t>(m) * ntot;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int mm = static_cast<int>(i / ntot), g = static_cast<int>(i % ntot);
    int sgi = 0;
    while (sgi + 1 < rs.nseg && g >= rs.row0[sgi + 1]) ++sgi;
    float v = 0.f;
    for (int z = 0; z < ks; ++z) v += part[z * total + i];
    store_y_rt(rs.y[sgi], ytype, static_cast<int64_t>(mm) * rs.ldy[sgi] + (g - rs.row0[sgi]), v);
  }
}

static int env_int(const char* name, int dflt) {
  const char* e = std::getenv(name);
  return e && e[0] ? std::atoi(e) : dflt;
}

static int sm_count() {
  int dev = 0, v = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) return 148;
  return v;
}

// K slices per tile: one CTA per SM, so a launch of `tiles` tiles split ks ways runs
// ceil(tiles * ks / sms) waves of 1/ks of the work each, plus a fixed cost per wave
// (pipeline fill, TMEM allocation, epilogue) taken as 8 k-blocks of work.
static int pick_fused_ksplit(int64_t tiles, int nkb, int64_t m, int64_t n, size_t part_bytes, int occ = 1) {
  const int forced = env_int("GGUFMM_FUSED_KSPLIT", -1);
  const int sms = sm_count() * occ;
  int best = 1;
  double best_cost = 1e30;
  for (int ks = 1; ks <= 16; ++ks) {
    if (ks > 1 && (nkb / ks < 4 || static_cast<size_t>(ks) * m * n * 4 > part_bytes)) break;
    const double waves = static_cast<double>((tiles * ks + sms - 1) / sms);
    const double cost = waves * (1.0 / ks + 8.0 / nkb);
    if (cost < best_cost * 0.999) best_cost = cost, best = ks;
    if (forced > 0 && ks == forced) return ks;
  }
  return forced == 0 ? 1 : best;
}

// The launch's segment table (tensor maps of each weight's headers and nibbles,
// outputs, tile and row offsets) and its copy for the K split's reduction.
static bool fill_segs(FusedSegs& sg, ReduceSegs& rs, int nseg, const void* const* q, const int64_t* n, int64_t k,
                      void* const* y, const int64_t* ldy) {
  const int64_t row_bytes = k / 256 * 144;
  memset(&sg, 0, sizeof(sg));
  memset(&rs, 0, sizeof(rs));
  sg.nseg = rs.nseg = nseg;
  sg.row_bytes = row_bytes;
  for (int i = 0; i < nseg; ++i) {
    if (!make_map_q(&sg.hdr[i], q[i], n[i], row_bytes, 16) || !make_map_q(&sg.qs[i], q[i], n[i], row_bytes, 64, CU_TENSOR_MAP_SWIZZLE_64B))
      return false;
    sg.y[i] = rs.y[i] = y[i];
    sg.ldy[i] = rs.ldy[i] = ldy[i];
    sg.n[i] = static_cast<int>(n[i]);
    sg.tile0[i + 1] = sg.tile0[i] + static_cast<int>((n[i] + kTileW - 1) / kTileW);
    sg.row0[i + 1] = rs.row0[i + 1] = sg.row0[i] + static_cast<int>(n[i]);
  }
  return true;
}

// zs_out != nullptr: every K slice (even a single one) leaves its fp32 partials in
// part_ws and no reduction is launched; *zs_out receives the slice count, for an
// epilogue pass (ffn_epilogue_kernel) that sums them.
template <int BN, int OCC>
static cudaError_t launch_fused_bn(int nseg, const void* const* q, const int64_t* n, const void* x16, int64_t m,
                                   int64_t k, void* const* y, int ytype, const int64_t* ldy, void* part_ws,
                                   size_t part_bytes, cudaStream_t st, int* zs_out = nullptr) {
  constexpr uint32_t kSmem = FusedTmemSmem<BN, OCC>::kTotal;
  FusedSegs sg;
  ReduceSegs rs;
  if (!fill_segs(sg, rs, nseg, q, n, k, y, ldy)) return cudaErrorInvalidValue;
  CUtensorMap mx;
  if (!make_map_f16(&mx, x16, m, k, BN)) return cudaErrorInvalidValue;
  auto fn = gemm_fused_q4k_tmem_kernel<BN, OCC>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(g_fused_attr_mu);
    if (!g_fused_attr_done.count({reinterpret_cast<const void*>(fn), dev})) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmem));
      if (e != cudaSuccess) return e;
      g_fused_attr_done.insert({reinterpret_cast<const void*>(fn), dev});
    }
  }
  const int64_t mt = (m + BN - 1) / BN, nt = sg.tile0[nseg], ntot = sg.row0[nseg];
  const int nkb = static_cast<int>(k / kFKB);
  const int ks = part_ws ? pick_fused_ksplit(mt * nt, nkb, m, ntot, part_bytes, OCC) : 1;
  const int kb_per = (nkb + ks - 1) / ks;
  const int zs = (nkb + kb_per - 1) / kb_per;  // slices actually used (each >= 1 k-block)
  float* part = (zs > 1 || zs_out) ? static_cast<float*>(part_ws) : nullptr;
  if (zs_out && (!part || part_bytes < static_cast<size_t>(zs) * m * ntot * 4)) return cudaErrorInvalidValue;
  dim3 grid(static_cast<unsigned>(mt), static_cast<unsigned>(nt), static_cast<unsigned>(zs));
  // programmatic dependent launch: the kernel waits for its predecessor itself
  // (pdl_wait before x, y and the partials) and streams its first weights before that
  e = pdl_launch(fn, grid, dim3(kFusedThreads), kSmem, st, sg, mx, ytype, static_cast<int>(m), static_cast<int>(k),
                 part, kb_per);
  if (zs_out) {
    *zs_out = zs;
    return e;
  }
  if (e != cudaSuccess || !part) return e;
  const int64_t total = m * ntot;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 8 * 148));
  return pdl_launch(fused_splitk_reduce_kernel, dim3(blocks), dim3(256), 0, st, static_cast<const float*>(part), zs,
                    static_cast<int>(m), rs, ytype);
}

// Two CTAs per SM (M <= 64, 256 TMEM columns each) where the launch has much work --
// (128-row tile, k-block) units -- so one CTA's pipeline fill and drain overlap the
// other's steady state and the waves are half as coarse (8B gate/up at M = 16: 45.2 ->
// 39.2 us, down 24.7 -> 23.1); the small launches (q/k/v, o) measured 1-7 % slower
// with it. GGUFMM_FUSED_OCC=1 / 2 forces one form.
template <int BN>
static cudaError_t launch_fused_dq(int nseg, const void* const* q, const int64_t* n, const void* x16, int64_t m,
                                   int64_t k, void* const* y, int ytype, const int64_t* ldy, void* part_ws,
                                   size_t part_bytes, cudaStream_t st, int* zs_out = nullptr) {
  static const int occ_env = env_int("GGUFMM_FUSED_OCC", 0);
  int64_t units = 0;
  for (int i = 0; i < nseg; ++i) units += (n[i] + kTileW - 1) / kTileW * (k / kFKB);
  const int occ = occ_env ? occ_env : (units >= 3000 ? 2 : 1);
  if constexpr (BN <= 64) {
    if (occ == 2)
      return launch_fused_bn<BN, 2>(nseg, q, n, x16, m, k, y, ytype, ldy, part_ws, part_bytes, st, zs_out);
  }
  return launch_fused_bn<BN, 1>(nseg, q, n, x16, m, k, y, ytype, ldy, part_ws, part_bytes, st, zs_out);
}

// nseg (1..4) Q4_K weights q[i] (16-byte aligned GGUF blocks [n[i], k/256*144]) times
// fp16 activations x16 [m, k] (row-major, 16-byte aligned) into y[i] [m, n[i]] with
// row stride ldy[i]. part_ws (256-byte aligned, part_bytes long, may be null) holds
// the fp32 partial sums when K is split across CTAs.
cudaError_t launch_gemm_fused_q4k_grouped(int nseg, const void* const* q, const int64_t* n, const void* x16,
                                          int64_t m, int64_t k, void* const* y, int ytype, const int64_t* ldy,
                                          void* part_ws, size_t part_bytes, cudaStream_t st) {
  if (nseg < 1 || nseg > kMaxFusedSegs) return cudaErrorInvalidValue;
  if (m <= 32) return launch_fused_dq<32>(nseg, q, n, x16, m, k, y, ytype, ldy, part_ws, part_bytes, st);
  if (m <= 64) return launch_fused_dq<64>(nseg, q, n, x16, m, k, y, ytype, ldy, part_ws, part_bytes, st);
  if (m <= 128) return launch_fused_dq<128>(nseg, q, n, x16, m, k, y, ytype, ldy, part_ws, part_bytes, st);
  // prefill: 256-token tiles; each CTA dequantizes its weight tile again for its token
  // tile, on the ALU while the tensor core works (a k-block's MMAs take about as long
  // as its dequantization), so the fp16 weight never goes through HBM
  return launch_fused_dq<256>(nseg, q, n, x16, m, k, y, ytype, ldy, part_ws, part_bytes, st);
}

// The fused GEMM leaving fp32 partials [zs][m][sum of n] in part_ws for an epilogue
// pass; *zs_out = the K slices.
cudaError_t launch_gemm_fused_q4k_partials(int nseg, const void* const* q, const int64_t* n, const void* x16,
                                           int64_t m, int64_t k, void* part_ws, size_t part_bytes, int* zs_out,
                                           cudaStream_t st) {
  if (nseg < 1 || nseg > kMaxFusedSegs) return cudaErrorInvalidValue;
  void* ys[kMaxFusedSegs] = {};
  int64_t lds[kMaxFusedSegs] = {};
  for (int i = 0; i < nseg; ++i) {
    ys[i] = part_ws;  // unused: every slice writes partials
    lds[i] = n[i];
  }
  if (m <= 32) return launch_fused_dq<32>(nseg, q, n, x16, m, k, ys, GGUFMM_F32, lds, part_ws, part_bytes, st, zs_out);
  if (m <= 64) return launch_fused_dq<64>(nseg, q, n, x16, m, k, ys, GGUFMM_F32, lds, part_ws, part_bytes, st, zs_out);
  if (m <= 128)
    return launch_fused_dq<128>(nseg, q, n, x16, m, k, ys, GGUFMM_F32, lds, part_ws, part_bytes, st, zs_out);
  return launch_fused_dq<256>(nseg, q, n, x16, m, k, ys, GGUFMM_F32, lds, part_ws, part_bytes, st, zs_out);
}

// The FFN epilogues, over fp32 partial sums part[ks][m][ntot] (ks K slices summed in
// order, so the result does not depend on CTA timing):
//   mode 0 (SwiGLU): ntot = 2n, gate in columns [0, n), up in [n, 2n):
//            y[mm, r] = silu(g) * u with silu(g) = g / (1 + e^-g) in fp32 -- the reference's
//            gelu_mul shader (shaders/generic/gelu_mul.wgsl:14-20);
//   mode 1 (residual): ntot = n, y[mm, r] = sum + resid[mm, r] (resid in y's dtype, row
//            stride ldr; it may be y itself) -- the reference's add shader after the o / down
//            projection (models/llama.py:335, 362).
// One rounding into y's dtype.
__global__ void ffn_epilogue_kernel(const float* __restrict__ part, int ks, int m, int n, int mode, const void* resid,
                                    int64_t ldr, void* y, int ytype, int64_t ldy) {
  pdl_trigger();
  pdl_wait();
  const int64_t ntot = mode == 0 ? 2 * static_cast<int64_t>(n) : n;
  const int64_t total = static_cast<int64_t>(m) * n, slice = static_cast<int64_t>(m) * ntot;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t mm = i / n, r = i - mm * n;
    float a = 0.f;
    for (int z = 0; z < ks; ++z) a += part[z * slice + mm * ntot + r];
    float v;
    if (mode == 0) {
      float u = 0.f;
      for (int z = 0; z < ks; ++z) u += part[z * slice + mm * ntot + n + r];
      v = a / (1.f + __expf(-a)) * u;
    } else {
      v = a + load_y_rt(resid, ytype, mm * ldr + r);
    }
    store_y_rt(y, ytype, mm * ldy + r, v);
  }
}

cudaError_t launch_ffn_epilogue(const float* part, int ks, int64_t m, int64_t n, int mode, const void* resid,
                                int64_t ldr, void* y, int ytype, int64_t ldy, cudaStream_t st) {
  const int64_t total = m * n;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 8 * 148));
  return pdl_launch(ffn_epilogue_kernel, dim3(blocks), dim3(256), 0, st, part, ks, static_cast<int>(m),
                    static_cast<int>(n), mode, resid, ldr, y, ytype, ldy);
}

cudaError_t launch_gemm_fused_q4k(const void* q, const void* x16, int64_t n, int64_t m, int64_t k, void* y, int ytype,
                                  int64_t ldy, void* part_ws, size_t part_bytes, cudaStream_t st) {
  return launch_gemm_fused_q4k_grouped(1, &q, &n, x16, m, k, &y, ytype, &ldy, part_ws, part_bytes, st);
}

cudaError_t gemm_fused_device_error(int* v, int clear, cudaStream_t st) { return tu_device_error(v, clear, st); }
cudaError_t gemm_fused_set_wait_limit(uint32_t polls) { return tu_set_wait_limit(polls); }

}  // namespace ggufmm
