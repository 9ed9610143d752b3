// tcgen05.cuh -- sm_100a tensor-core (tcgen05 / TMEM) and TMA helpers shared by
// the GEMM kernels: UMMA shared-memory and instruction descriptors, 2-D tiled TMA
// loads, MMA issue / commit, TMEM loads, and the host-side tensor-map encoder.
#pragma once

#include <mutex>

#include "common.cuh"

namespace ggufmm {

constexpr int kTileW = 128;  // weight rows per CTA tile (MMA M)
constexpr int kBK = 64;      // k elements per 128-byte swizzle row of fp16

__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t saddr) {
  // K-major operand, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart.
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);         // start address
  d |= static_cast<uint64_t>(1) << 16;                          // leading byte offset (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;                  // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;                          // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                          // layout: SWIZZLE_128B
  return d;
}

template <int BN>
__device__ __forceinline__ constexpr uint32_t umma_idesc_f16() {
  // D = f32 (bits 4-5 = 1), A = B = f16 (0), both K-major, N>>3 at bit 17, M>>4 at bit 24.
  return (1u << 4) | (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(kTileW >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The same load without the wait: several may be in flight before tmem_wait_ld.
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// One epilogue warp's 32 accumulator lanes (weight row nrow) x BN columns (tokens
// m0..) into y[token, nrow] of type YT: CH columns per TMEM wait (the loads'
// latency is paid once per chunk), typed stores.
// BN: columns this warp drains (a multiple of 16); CHMAX caps the chunk (registers).
template <int BN, int YT, int CHMAX = 64>
__device__ __forceinline__ void drain_tile(uint32_t tbase, void* y, int64_t ldy, int m0, int m, int nrow, int n) {
  constexpr int CH = BN % 64 == 0 && CHMAX >= 64 ? 64 : BN % 32 == 0 && CHMAX >= 32 ? 32 : 16;
  const bool row_ok = nrow < n;
  const int cols = min(BN, m - m0);  // live token columns of this tile
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += CH) {
    uint32_t r[CH];
#pragma unroll
    for (int h = 0; h < CH; h += 16) tmem_ld16_async(tbase + c0 + h, r + h);
    tmem_wait_ld();
    if (row_ok) {
      const int64_t base = static_cast<int64_t>(m0 + c0) * ldy + nrow;
      if (c0 + CH <= cols) {
#pragma unroll
        for (int j = 0; j < CH; ++j) store_y<YT>(y, base + j * ldy, __uint_as_float(r[j]));
      } else {
#pragma unroll
        for (int j = 0; j < CH; ++j)
          if (c0 + j < cols) store_y<YT>(y, base + j * ldy, __uint_as_float(r[j]));
      }
    }
  }
}



// ---- host side --------------------------------------------------------------
typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline PFN_encodeTiled get_encode_fn() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

// fp16 row-major [rows, k] tensor, box = 64 (k) x box_rows, 128-byte swizzle.
inline bool make_map_f16(CUtensorMap* map, const void* base, int64_t rows, int64_t k, int box_rows) {
  PFN_encodeTiled enc = get_encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(k) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}


}  // namespace ggufmm
