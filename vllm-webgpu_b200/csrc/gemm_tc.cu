// gemm_tc.cu -- prefill / batched GEMM on the sm_100a 5th-generation tensor
// cores: Y[m, n] = sum_k X[m, k] W[n, k] with fp16 operands (W is the GGUF
// weight dequantized in fp32 and rounded once to fp16, X the activations cast
// to fp16) and fp32 accumulation in tensor memory (TMEM).
//
// Replaces matmul_quant_mr4.wgsl:77-131 of maci0/vllm-webgpu (one thread per
// 4x1 output tile, never dispatched) and the token-at-a-time prefill of
// run_inference.py:323-350.
//
// One CTA computes a 128 (weight rows) x BN (tokens) tile; the weight rows are
// the MMA's M dimension ("swap AB"), so decode-sized token counts still fill
// the 128-lane datapath. Warp roles (192 threads):
//   warp 0      TMA producer: 2-D tiled loads (128-byte swizzle) of the W and X
//               k-blocks into a `kStages`-deep shared-memory ring; completion
//               via mbarrier transaction counts.
//   warp 1      allocates TMEM; one elected lane issues tcgen05.mma
//               (kind::f16, M=128, N=BN, K=16) per 16-wide k-step, commits
//               each stage back to the producer, and finally the accumulator
//               to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld 32x32b from TMEM (each warp owns the 32
//               TMEM lanes its warp-in-quad index selects), transpose on the
//               fly, coalesced stores of Y.
// Every TMA load is a plain (single-CTA) load of this GPU's own memory.
#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

#include "tcgen05.cuh"

namespace ggufmm {

// Optional peer outputs: the tile's values are stored into `world` [m, ldy] outputs
// (this GPU's and its peers', mapped here over NVLink) at column col0 + row -- the
// N-split GEMM's all-gather done by the epilogue itself, overlapped with the MMAs of
// later tiles. world 0: the single output y.
struct PeerOut {
  uint64_t y[8];
  int world;
  int64_t col0;
  int vec;  // 16-bit outputs, 16-byte aligned rows and bases: staged 16-byte peer stores
};

__device__ __forceinline__ void store_out(void* y, const PeerOut& po, int ytype, int64_t mm, int64_t ldy, int nrow,
                                          float v) {
  if (po.world == 0) {
    store_y_rt(y, ytype, mm * ldy + nrow, v);
    return;
  }
  for (int p = 0; p < po.world; ++p) store_y_rt(reinterpret_cast<void*>(po.y[p]), ytype, mm * ldy + po.col0 + nrow, v);
}

// AND of a predicate over the 4 epilogue warps (named barrier 1, 128 threads).
__device__ __forceinline__ bool epi_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbarrier.red.and.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}

// tcgen05.alloc takes a power of two >= 32 columns.
__host__ __device__ constexpr uint32_t tmem_cols_pow2(uint32_t c) {
  uint32_t p = 32;
  while (p < c) p <<= 1;
  return p;
}

// Tail split of the persistent GEMM. The first `whole` tiles run whole, as the
// CTAs' first full waves; each of the remaining tiles is cut along K into
// `slices` pieces of `kper` k-blocks, one piece per CTA, so the last wave lasts
// 1/slices of a tile instead of a whole one. A piece leaves its fp32 partial tile
// in part[piece][column][row] and gemm_tail_reduce_kernel adds the slices in order.
struct TailSplit {
  float* part;
  int whole;
  int slices;  // 1: no split
  int kper;
};

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr uint32_t kABytes = kTileW * kBK * 2;  // 16 KB
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kBarOff = STAGES * kStageBytes;
  // the peer epilogue's transpose tile: 16 tokens x 128 rows of 16-bit outputs
  static constexpr uint32_t kEpiOff = (kBarOff + (2 * STAGES + 6) * 8 + 16 + 15) / 16 * 16;
  static constexpr uint32_t kTotal = kEpiOff + 4 * 16 * 32 * 2 + 1024;  // + alignment slack
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                   void* __restrict__ y, int ytype, int64_t ldy, int n, int m, int k, const PeerOut po,
                   const TailSplit) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  // 128-byte swizzled tiles need 1024-byte aligned bases
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // token tiles vary fastest: the CTAs that share one weight tile run together,
  // so the weight (the large operand) streams from HBM once and the rest hit L2
  const int m0 = blockIdx.x * BN, n0 = blockIdx.y * kTileW;
  const int nk = (k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_d = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % STAGES;
        if (!mbar_wait(&empty[s], ((kb / STAGES) & 1) ^ 1)) break;
        uint8_t* a_dst = smem + s * L::kStageBytes;
        uint8_t* b_dst = a_dst + L::kABytes;
        mbar_arrive_expect_tx(&full[s], L::kStageBytes);
        tma_load_2d(a_dst, &tmap_w, kb * kBK, n0, &full[s]);
        tma_load_2d(b_dst, &tmap_x, kb * kBK, m0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16<BN>();
      bool ok = true;
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % STAGES;
        ok = mbar_wait(&full[s], (kb / STAGES) & 1);
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_addr = smem_u32(smem + s * L::kStageBytes);
        const uint32_t b_addr = a_addr + L::kABytes;
        const uint64_t adesc = umma_smem_desc(a_addr), bdesc = umma_smem_desc(b_addr);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk) {
          // advance 16 fp16 = 32 bytes along K inside the swizzle atom
          umma_f16(tmem_d, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
      }
      umma_commit(accum);  // all MMAs issued so far complete -> accumulator ready
    }
  } else {
    // epilogue warps 2..5: TMEM lanes 32*(warp%4) .. +31 = weight rows
    const int quad = warp & 3;
    const bool ok = mbar_wait(accum, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok) {
      const int nrow = n0 + quad * 32 + lane;
      const uint32_t tbase = tmem_d + (static_cast<uint32_t>(quad * 32) << 16);
      if (po.world == 0 && ytype == GGUFMM_BF16) {
        drain_tile<BN, GGUFMM_BF16>(tbase, y, ldy, m0, m, nrow, n);
      } else if (po.world == 0 && ytype == GGUFMM_F32) {
        drain_tile<BN, GGUFMM_F32>(tbase, y, ldy, m0, m, nrow, n);
      } else if (po.world == 0) {
        drain_tile<BN, GGUFMM_F16>(tbase, y, ldy, m0, m, nrow, n);
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(tbase + c0, r);
          if (nrow < n) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int mm = m0 + c0 + j;
              if (mm < m) store_out(y, po, ytype, mm, ldy, nrow, __uint_as_float(r[j]));
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(BN) : "memory");
  }
}

// Persistent variant: one CTA per SM walks the tiles (token tiles fastest) and
// keeps TWO accumulators in TMEM (2 x BN columns), so the epilogue warps drain
// tile i while the MMA warp already accumulates tile i+1, and TMEM allocation,
// barrier set-up and pipeline fill are paid once per CTA instead of per tile.
//   tfull[b]   MMA warp -> epilogue: accumulator b holds a finished tile
//   tempty[b]  epilogue (4 warps) -> MMA warp: accumulator b has been read
template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_persistent_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                              void* __restrict__ y, int ytype, int64_t ldy, int n, int m, int k,
                              const PeerOut po, const TailSplit ts) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  // the two accumulators start half the (power-of-two) allocation apart
  constexpr uint32_t kAccStride = tmem_cols_pow2(2 * BN) / 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mtiles = (m + BN - 1) / BN, ntiles = (n + kTileW - 1) / kTileW;
  const int tiles = mtiles * ntiles;
  const int nk = (k + kBK - 1) / kBK;
  const int bid = static_cast<int>(blockIdx.x), grid = static_cast<int>(gridDim.x);
  // work items of this CTA: whole tiles bid, bid + grid, ... below ts.whole, then
  // (tail split) piece bid of the remaining tiles
  const int whole = ts.slices > 1 ? ts.whole : tiles;
  const int my_whole = whole > bid ? (whole - 1 - bid) / grid + 1 : 0;
  const bool has_piece = ts.slices > 1 && bid < (tiles - whole) * ts.slices;
  const int my_tiles = my_whole + (has_piece ? 1 : 0);
  // item i -> token / weight tile origin, k-block range, piece index (-1: whole tile)
  auto item = [&](int i, int& m0, int& n0, int& kb0, int& kb1) -> int {
    int t = bid + i * grid, piece = -1;
    kb0 = 0;
    kb1 = nk;
    if (i >= my_whole) {
      piece = bid;
      t = whole + bid / ts.slices;
      kb0 = (bid % ts.slices) * ts.kper;
      kb1 = min(nk, kb0 + ts.kper);
    }
    m0 = (t % mtiles) * BN;
    n0 = (t / mtiles) * kTileW;
    return piece;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_w)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_x)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols_pow2(2 * BN))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_d = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int q = 0;  // running k-block index over all of this CTA's tiles
      bool ok = true;
      for (int i = 0; i < my_tiles && ok; ++i) {
        int m0, n0, kb0, kb1;
        item(i, m0, n0, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++q) {
          const int s = q % STAGES;
          if (!mbar_wait(&empty[s], ((q / STAGES) & 1) ^ 1)) {
            ok = false;
            break;
          }
          uint8_t* a_dst = smem + s * L::kStageBytes;
          uint8_t* b_dst = a_dst + L::kABytes;
          mbar_arrive_expect_tx(&full[s], L::kStageBytes);
          tma_load_2d(a_dst, &tmap_w, kb * kBK, n0, &full[s]);
          tma_load_2d(b_dst, &tmap_x, kb * kBK, m0, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16<BN>();
      int q = 0;
      bool ok = true;
      for (int i = 0; i < my_tiles && ok; ++i) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait(&tempty[b], static_cast<uint32_t>(((i >> 1) - 1) & 1))) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem_d + static_cast<uint32_t>(b) * kAccStride;
        int m0, n0, kb0, kb1;
        item(i, m0, n0, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++q) {
          const int s = q % STAGES;
          if (!mbar_wait(&full[s], (q / STAGES) & 1)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_addr = smem_u32(smem + s * L::kStageBytes);
          const uint32_t b_addr = a_addr + L::kABytes;
          const uint64_t adesc = umma_smem_desc(a_addr), bdesc = umma_smem_desc(b_addr);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(acc, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&tfull[b]);  // this tile's MMAs complete -> accumulator b ready
      }
    }
  } else {
    // epilogue warps 2..5: TMEM lanes 32*(warp%4) .. +31 = weight rows
    const int quad = warp & 3;
    for (int i = 0; i < my_tiles; ++i) {
      const int b = i & 1;
      int m0, n0, kb0, kb1;
      const int piece = item(i, m0, n0, kb0, kb1);
      bool okw = mbar_wait(&tfull[b], static_cast<uint32_t>((i >> 1) & 1));
      if (po.world > 0) okw = epi_all(okw);  // the peer epilogue syncs the 4 warps: leave together
      if (!okw) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int nrow = n0 + quad * 32 + lane;
      const uint32_t tbase = tmem_d + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(b) * kAccStride;
      if (piece >= 0) {
        // partial tile, column-major: a warp's 32 rows are one 128-byte store
        float* pp = ts.part + static_cast<int64_t>(piece) * BN * kTileW + quad * 32 + lane;
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(tbase + c0, r);
#pragma unroll
          for (int j = 0; j < 16; ++j) pp[(c0 + j) * kTileW] = __uint_as_float(r[j]);
        }
      } else if (po.world == 0 && ytype == GGUFMM_BF16) {
        drain_tile<BN, GGUFMM_BF16>(tbase, y, ldy, m0, m, nrow, n);
      } else if (po.world == 0 && ytype == GGUFMM_F32) {
        drain_tile<BN, GGUFMM_F32>(tbase, y, ldy, m0, m, nrow, n);
      } else if (po.world == 0) {
        drain_tile<BN, GGUFMM_F16>(tbase, y, ldy, m0, m, nrow, n);
      } else if (po.vec && m0 + BN <= m && n0 + kTileW <= n) {
        // all-gather in the epilogue, whole tile: 16 tokens at a time through a
        // transpose tile in shared memory, so each lane stores 16 contiguous bytes (8
        // outputs of one token) to every GPU -- a warp instruction moves 512 bytes per
        // GPU instead of 64 with one 2-byte store per lane. The condition is the same
        // for the 4 epilogue warps (one tile), so all of them reach the barriers.
        // the 4 epilogue warps fill one [16 tokens][128 rows] tile together (named barrier
        // 1), so each token's 256 bytes go out as 16 contiguous 16-byte stores
        uint16_t* tt = reinterpret_cast<uint16_t*>(smem + L::kEpiOff);
        const bool bf = ytype == GGUFMM_BF16;
        const int et = quad * 32 + lane;  // 0..127 over the epilogue warps
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(tbase + c0, r);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float v = __uint_as_float(r[j]);
            tt[j * kTileW + et] = bf ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : __half_as_ushort(__float2half_rn(v));
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int ch = et + 128 * h, jj = ch >> 4, qq = ch & 15;
            const uint4 v = *reinterpret_cast<const uint4*>(tt + jj * kTileW + qq * 8);
            const int64_t off = static_cast<int64_t>(m0 + c0 + jj) * ldy + po.col0 + n0 + qq * 8;
            for (int p = 0; p < po.world; ++p) *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(po.y[p]) + off) = v;
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
      } else {
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          uint32_t r[16];
          tmem_ld16(tbase + c0, r);
          if (nrow < n) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int mm = m0 + c0 + j;
              if (mm < m) store_out(y, po, ytype, mm, ldy, nrow, __uint_as_float(r[j]));
            }
          }
        }
      }
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(tmem_cols_pow2(2 * BN)) : "memory");
  }
}

// ---- host side --------------------------------------------------------------
static std::mutex g_gemm_attr_mu;
static std::set<std::pair<const void*, int>> g_gemm_attr_done;

static int device_sms() {
  static const int sms = [] {
    int dev = 0, v = 148;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      v = 148;
    return v;
  }();
  return sms;
}

constexpr int kTailMinKb = 8;  // k-blocks per piece at least (pipeline fill amortised)

// Tail split for `tiles` tiles of width bn on `sms` CTAs (slices 1: none). With
// part_bytes < 0 the workspace is not limiting.
static TailSplit tail_plan(int64_t tiles, int nk, int sms, int bn, int64_t part_bytes) {
  TailSplit ts{nullptr, static_cast<int>(tiles), 1, nk};
  const int64_t rest = tiles % sms;
  if (rest == 0) return ts;
  int64_t sl = std::min<int64_t>(sms / rest, nk / kTailMinKb);
  const int64_t piece_bytes = static_cast<int64_t>(bn) * kTileW * 4;
  if (part_bytes >= 0) sl = std::min<int64_t>(sl, part_bytes / (rest * piece_bytes));
  if (sl < 2) return ts;
  ts.kper = (nk + static_cast<int>(sl) - 1) / static_cast<int>(sl);
  ts.slices = (nk + ts.kper - 1) / ts.kper;  // every piece non-empty
  if (ts.slices < 2) return TailSplit{nullptr, static_cast<int>(tiles), 1, nk};
  ts.whole = static_cast<int>(tiles - rest);
  return ts;
}

// y[m0 + c, n0 + r] = sum over s (in order) of part[(t * slices + s) * bn + c][r] for
// the split tiles t (the tail of the persistent GEMM).
__global__ void __launch_bounds__(256) gemm_tail_reduce_kernel(const float* __restrict__ part, int whole, int rtiles,
                                                               int slices, int bn, int mtiles, int n, int m,
                                                               void* __restrict__ y, int ytype, int64_t ldy,
                                                               const PeerOut po) {
  const int64_t per_tile = static_cast<int64_t>(bn) * kTileW;
  const int64_t total = rtiles * per_tile;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int j = static_cast<int>(i / per_tile);
    const int64_t e = i - j * per_tile;
    const int c = static_cast<int>(e / kTileW), r = static_cast<int>(e % kTileW);
    const int t = whole + j;
    const int mm = (t % mtiles) * bn + c, nrow = (t / mtiles) * kTileW + r;
    if (mm >= m || nrow >= n) continue;
    const float* pp = part + static_cast<int64_t>(j) * slices * per_tile + e;
    float v = 0.f;
    for (int s = 0; s < slices; ++s) v += pp[s * per_tile];
    store_out(y, po, ytype, mm, ldy, nrow, v);
  }
}

template <int BN, int STAGES, bool PERSIST = false>
static cudaError_t launch_gemm_bn(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k, void* y,
                                  int ytype, int64_t ldy, cudaStream_t st, const PeerOut& po, float* part,
                                  size_t part_bytes) {
  using L = GemmSmem<BN, STAGES>;
  CUtensorMap mw, mx;
  if (!make_map_f16(&mw, w16, n, k, kTileW) || !make_map_f16(&mx, x16, m, k, BN)) return cudaErrorInvalidValue;
  auto fn = PERSIST ? gemm_tc_persistent_kernel<BN, STAGES> : gemm_tc_kernel<BN, STAGES>;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  {
    std::lock_guard<std::mutex> lk(g_gemm_attr_mu);
    if (!g_gemm_attr_done.count({reinterpret_cast<const void*>(fn), dev})) {
      e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(L::kTotal));
      if (e != cudaSuccess) return e;
      g_gemm_attr_done.insert({reinterpret_cast<const void*>(fn), dev});
    }
  }
  const int64_t mtiles = (m + BN - 1) / BN, tiles = mtiles * ((n + kTileW - 1) / kTileW);
  const int nk = static_cast<int>((k + kBK - 1) / kBK);
  dim3 grid(static_cast<unsigned>(mtiles), static_cast<unsigned>((n + kTileW - 1) / kTileW));
  TailSplit ts{nullptr, static_cast<int>(tiles), 1, nk};
  if (PERSIST) {
    const int sms = device_sms();
    if (part) ts = tail_plan(tiles, nk, sms, BN, static_cast<int64_t>(part_bytes));
    ts.part = part;
    grid = dim3(static_cast<unsigned>(ts.slices > 1 ? sms : std::min<int64_t>(tiles, sms)));
  }
  fn<<<grid, 192, L::kTotal, st>>>(mw, mx, y, ytype, ldy, static_cast<int>(n), static_cast<int>(m),
                                   static_cast<int>(k), po, ts);
  e = cudaGetLastError();
  if (e != cudaSuccess || ts.slices < 2) return e;
  const int rtiles = static_cast<int>(tiles) - ts.whole;
  const int64_t total = static_cast<int64_t>(rtiles) * BN * kTileW;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4 * 148));
  gemm_tail_reduce_kernel<<<blocks, 256, 0, st>>>(part, ts.whole, rtiles, ts.slices, BN, static_cast<int>(mtiles),
                                                  static_cast<int>(n), static_cast<int>(m), y, ytype, ldy, po);
  return cudaGetLastError();
}

cudaError_t gemm_device_error(int* v, int clear, cudaStream_t st) { return tu_device_error(v, clear, st); }
cudaError_t gemm_set_wait_limit(uint32_t polls) { return tu_set_wait_limit(polls); }

// Token-tile width of the persistent GEMM. Every CTA runs whole tiles, so the
// last wave of ceil(tiles / SMs) is partly idle unless the tail is split along K
// (tail_plan, when the caller gives partial-sum space). The width minimises
// waves x (width + 192), with the tail counted as 1/slices + 0.15 of a wave; the 192
// stands for a tile's fixed cost (accumulator hand-off, pipeline fill, and a
// narrower tile's extra weight-tile fetches per flop). Without the split the
// constant was fitted on B200 over K = 4096, N = 1792..14336, M = 512..8192
// (Q4_K and Q6_K): the pick was the fastest width in every case, e.g. N = 3584,
// M = 512 runs 128-wide in 49.9 us against 59.1 us 256-wide, while N = 14336,
// M = 2048 stays 256-wide (253 us; 160-wide 266.8 us).
// GGUFMM_GEMM_BN = 128|160|192|224|256 forces a width.
static int persistent_bn(int64_t n, int64_t m, int64_t k, bool split) {
  static const int forced = [] {
    const char* e = std::getenv("GGUFMM_GEMM_BN");
    return e ? std::atoi(e) : 0;
  }();
  if (forced == 128 || forced == 160 || forced == 192 || forced == 224 || forced == 256) return forced;
  const int sms = device_sms();
  const int64_t ntiles = (n + kTileW - 1) / kTileW;
  const int nk = static_cast<int>((k + kBK - 1) / kBK);
  int best = 256;
  double best_cost = -1;
  for (int bn : {256, 224, 192, 160, 128}) {
    const int64_t tiles = ((m + bn - 1) / bn) * ntiles;
    const TailSplit ts = split ? tail_plan(tiles, nk, sms, bn, -1) : TailSplit{nullptr, 0, 1, nk};
    // a split tail also pays its partial-tile stores and the reduce pass (~0.15 wave)
    const double waves = ts.slices > 1 ? static_cast<double>(tiles / sms) + 1.0 / ts.slices + 0.15
                                       : static_cast<double>((tiles + sms - 1) / sms);
    const double cost = waves * (bn + 192);
    if (best_cost < 0 || cost < best_cost * 0.999) best = bn, best_cost = cost;
  }
  return best;
}

// Bytes of fp32 partial sums the persistent GEMM's tail split uses for this shape
// on the current device (0: no split).
size_t gemm_tail_bytes(int64_t n, int64_t m, int64_t k) {
  if (m <= 128) return 0;
  const int bn = persistent_bn(n, m, k, true);
  const int64_t tiles = ((m + bn - 1) / bn) * ((n + kTileW - 1) / kTileW);
  const TailSplit ts = tail_plan(tiles, static_cast<int>((k + kBK - 1) / kBK), device_sms(), bn, -1);
  if (ts.slices < 2) return 0;
  return static_cast<size_t>(tiles - ts.whole) * ts.slices * bn * kTileW * 4;
}

// Tensor-core GEMM on fp16 operands already in device memory:
// w16 [n, k], x16 [m, k] (both row-major, 16-byte aligned, k % 8 == 0).
static cudaError_t launch_gemm_f16_po(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k, void* y,
                                      int ytype, int64_t ldy, cudaStream_t st, const PeerOut& po, float* part,
                                      size_t part_bytes) {
  if (m <= 32) return launch_gemm_bn<32, 8>(w16, x16, n, m, k, y, ytype, ldy, st, po, nullptr, 0);
  if (m <= 64) return launch_gemm_bn<64, 8>(w16, x16, n, m, k, y, ytype, ldy, st, po, nullptr, 0);
  if (m <= 128) return launch_gemm_bn<128, 6>(w16, x16, n, m, k, y, ytype, ldy, st, po, nullptr, 0);
  static const bool persist = [] {
    const char* e = std::getenv("GGUFMM_GEMM_PERSIST");
    return !(e && e[0] == '0');
  }();
  if (!persist) return launch_gemm_bn<256, 4>(w16, x16, n, m, k, y, ytype, ldy, st, po, nullptr, 0);
  static const bool split = [] {
    const char* e = std::getenv("GGUFMM_GEMM_TAIL");
    return !(e && e[0] == '0');
  }();
  if (!split) part = nullptr;
  switch (persistent_bn(n, m, k, part != nullptr)) {
    case 224: return launch_gemm_bn<224, 5, true>(w16, x16, n, m, k, y, ytype, ldy, st, po, part, part_bytes);
    case 192: return launch_gemm_bn<192, 5, true>(w16, x16, n, m, k, y, ytype, ldy, st, po, part, part_bytes);
    case 160: return launch_gemm_bn<160, 6, true>(w16, x16, n, m, k, y, ytype, ldy, st, po, part, part_bytes);
    case 128: return launch_gemm_bn<128, 6, true>(w16, x16, n, m, k, y, ytype, ldy, st, po, part, part_bytes);
    default: return launch_gemm_bn<256, 4, true>(w16, x16, n, m, k, y, ytype, ldy, st, po, part, part_bytes);
  }
}

// part (fp32, part_bytes long; may be null): partial sums for the tail split.
cudaError_t launch_gemm_f16(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k, void* y, int ytype,
                            int64_t ldy, cudaStream_t st, float* part, size_t part_bytes) {
  return launch_gemm_f16_po(w16, x16, n, m, k, y, ytype, ldy, st, PeerOut{}, part, part_bytes);
}

// The same GEMM storing every output value into `world` outputs (all GPUs' [m, ldy]
// buffers, peers' mapped over NVLink) at column col0 + row.
cudaError_t launch_gemm_f16_peers(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k,
                                  void* const* ys, int world, int64_t col0, int ytype, int64_t ldy, cudaStream_t st,
                                  float* part, size_t part_bytes) {
  if (world < 1 || world > 8) return cudaErrorInvalidValue;
  PeerOut po{};
  for (int i = 0; i < world; ++i) po.y[i] = reinterpret_cast<uint64_t>(ys[i]);
  po.world = world;
  po.col0 = col0;
  bool vec = ytype != GGUFMM_F32 && ldy % 8 == 0 && col0 % 8 == 0;
  for (int i = 0; i < world; ++i) vec = vec && (po.y[i] & 15) == 0;
  po.vec = vec ? 1 : 0;
  return launch_gemm_f16_po(w16, x16, n, m, k, ys[0], ytype, ldy, st, po, part, part_bytes);
}

}  // namespace ggufmm
