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
};

__device__ __forceinline__ void store_out(void* y, const PeerOut& po, int ytype, int64_t mm, int64_t ldy, int nrow,
                                          float v) {
  if (po.world == 0) {
    store_y_rt(y, ytype, mm * ldy + nrow, v);
    return;
  }
  for (int p = 0; p < po.world; ++p) store_y_rt(reinterpret_cast<void*>(po.y[p]), ytype, mm * ldy + po.col0 + nrow, v);
}

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr uint32_t kABytes = kTileW * kBK * 2;  // 16 KB
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kBarOff = STAGES * kStageBytes;
  static constexpr uint32_t kTotal = kBarOff + (2 * STAGES + 6) * 8 + 16 + 1024;  // + alignment slack
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(192, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                   void* __restrict__ y, int ytype, int64_t ldy, int n, int m, int k,
                              const PeerOut po) {
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
                              const PeerOut po) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mtiles = (m + BN - 1) / BN, ntiles = (n + kTileW - 1) / kTileW;
  const int tiles = mtiles * ntiles;
  const int nk = (k + kBK - 1) / kBK;
  const int my_tiles = tiles > static_cast<int>(blockIdx.x) ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

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
                 "r"(2 * BN)
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
        const int t = blockIdx.x + i * gridDim.x;
        const int m0 = (t % mtiles) * BN, n0 = (t / mtiles) * kTileW;
        for (int kb = 0; kb < nk; ++kb, ++q) {
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
        const uint32_t acc = tmem_d + static_cast<uint32_t>(b * BN);
        for (int kb = 0; kb < nk; ++kb, ++q) {
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
            umma_f16(acc, adesc + 2 * kk, bdesc + 2 * kk, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
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
      const int t = blockIdx.x + i * gridDim.x;
      const int m0 = (t % mtiles) * BN, n0 = (t / mtiles) * kTileW;
      if (!mbar_wait(&tfull[b], static_cast<uint32_t>((i >> 1) & 1))) break;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int nrow = n0 + quad * 32 + lane;
      const uint32_t tbase = tmem_d + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(b * BN);
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
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(2 * BN) : "memory");
  }
}

// ---- host side --------------------------------------------------------------
static std::mutex g_gemm_attr_mu;
static std::set<std::pair<const void*, int>> g_gemm_attr_done;

template <int BN, int STAGES, bool PERSIST = false>
static cudaError_t launch_gemm_bn(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k, void* y,
                                  int ytype, int64_t ldy, cudaStream_t st, const PeerOut& po = PeerOut{}) {
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
  dim3 grid(static_cast<unsigned>((m + BN - 1) / BN), static_cast<unsigned>((n + kTileW - 1) / kTileW));
  if (PERSIST) {
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    grid = dim3(static_cast<unsigned>(std::min<int64_t>(static_cast<int64_t>(grid.x) * grid.y, sms)));
  }
  fn<<<grid, 192, L::kTotal, st>>>(mw, mx, y, ytype, ldy, static_cast<int>(n), static_cast<int>(m),
                                   static_cast<int>(k), po);
  return cudaGetLastError();
}

cudaError_t gemm_device_error(int* v, int clear, cudaStream_t st) { return tu_device_error(v, clear, st); }
cudaError_t gemm_set_wait_limit(uint32_t polls) { return tu_set_wait_limit(polls); }

// Tensor-core GEMM on fp16 operands already in device memory:
// w16 [n, k], x16 [m, k] (both row-major, 16-byte aligned, k % 8 == 0).
static cudaError_t launch_gemm_f16_po(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k, void* y,
                                      int ytype, int64_t ldy, cudaStream_t st, const PeerOut& po) {
  if (m <= 32) return launch_gemm_bn<32, 8>(w16, x16, n, m, k, y, ytype, ldy, st, po);
  if (m <= 64) return launch_gemm_bn<64, 8>(w16, x16, n, m, k, y, ytype, ldy, st, po);
  if (m <= 128) return launch_gemm_bn<128, 6>(w16, x16, n, m, k, y, ytype, ldy, st, po);
  static const bool persist = [] {
    const char* e = std::getenv("GGUFMM_GEMM_PERSIST");
    return !(e && e[0] == '0');
  }();
  if (persist) return launch_gemm_bn<256, 4, true>(w16, x16, n, m, k, y, ytype, ldy, st, po);
  return launch_gemm_bn<256, 4>(w16, x16, n, m, k, y, ytype, ldy, st, po);
}

cudaError_t launch_gemm_f16(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k, void* y, int ytype,
                            int64_t ldy, cudaStream_t st) {
  return launch_gemm_f16_po(w16, x16, n, m, k, y, ytype, ldy, st, PeerOut{});
}

// The same GEMM storing every output value into `world` outputs (all GPUs' [m, ldy]
// buffers, peers' mapped over NVLink) at column col0 + row.
cudaError_t launch_gemm_f16_peers(const void* w16, const void* x16, int64_t n, int64_t m, int64_t k,
                                  void* const* ys, int world, int64_t col0, int ytype, int64_t ldy, cudaStream_t st) {
  if (world < 1 || world > 8) return cudaErrorInvalidValue;
  PeerOut po{};
  for (int i = 0; i < world; ++i) po.y[i] = reinterpret_cast<uint64_t>(ys[i]);
  po.world = world;
  po.col0 = col0;
  return launch_gemm_f16_po(w16, x16, n, m, k, ys[0], ytype, ldy, st, po);
}

}  // namespace ggufmm
