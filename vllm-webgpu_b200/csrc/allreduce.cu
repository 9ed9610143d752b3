// allreduce.cu -- one-shot all-reduce (sum) of a small fp32 vector over NVLink peer
// memory, for the tensor-parallel decode step's all-reduces (the o and down
// projections' partials, M x hidden fp32: 16 KB at M = 1), where a library
// collective spends most of its time in latency; and a device-side barrier.
//
// Every rank owns one exchange buffer, mapped into every other rank (symmetric
// memory):
//   [header: flag[src rank][cta] u32 (written by the peers), gen[cta] u32 (own)]
//   [data: 2 parities x world source ranks x n floats]
// A call runs kArCtas(n) CTAs; CTA c owns the 1024-value chunk c of the vector. Per
// call and CTA, on every rank ("push"):
//   1. gen = own gen[c] + 1 (device memory: the call can be captured in a CUDA graph
//      and replayed, no host-side epoch);
//   2. store the chunk of `in` into slot [gen & 1][rank] of EVERY rank's buffer (peer
//      stores over NVLink, 16 bytes per thread);
//   3. system-scope fence, then release flag[rank][c] = gen in every rank's buffer;
//   4. bounded acquire-wait on the LOCAL flags[src][c] >= gen of every source;
//   5. out chunk = sum over sources in rank order of the local slots (+ resid): the
//      same bits on every rank.
// Two parities suffice: a rank reaches call gen + 2 (and overwrites a peer's slot of
// parity gen & 1) only after every peer has flagged gen + 1, which each does after
// its reads of call gen. n = 0 is a barrier: every rank's earlier work on its stream
// (stores into peers' memory included) is complete and visible before any rank
// returns. A peer that never publishes makes the wait give up after the bounded poll
// count: the status word gets kErrWaitTimeout and out is not written. No multicast,
// no NVLS: plain peer stores and local loads.
#include <cstdlib>

#include "common.cuh"

namespace ggufmm {

namespace {

constexpr int kArThreads = 256;
constexpr int kArChunk = kArThreads * 4;  // floats per CTA
constexpr int kArMaxCtas = 64;
constexpr int64_t kArMaxN = static_cast<int64_t>(kArChunk) * kArMaxCtas;  // 65536 floats
constexpr int kArHeader = 8 * kArMaxCtas * 4 + kArMaxCtas * 4;           // flags + gens
constexpr int kArDataOff = (kArHeader + 255) / 256 * 256;

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct ArArgs {
  uint64_t buf[8];  // every rank's exchange buffer, as mapped on this GPU
  int world, rank;
  int64_t n;
  const float* in;
  float* out;
  const float* resid;  // optional, same layout as out
};

__global__ void __launch_bounds__(kArThreads) allreduce_push_kernel(const ArArgs a) {
  __shared__ uint32_t s_gen;
  __shared__ int s_ok;
  const int c = blockIdx.x;
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.buf[a.rank]);
  uint32_t* my_gen = reinterpret_cast<uint32_t*>(mine + 8 * kArMaxCtas * 4) + c;
  // the inputs (and the stores of earlier kernels, for the barrier) come before this
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) s_gen = *reinterpret_cast<volatile uint32_t*>(my_gen) + 1u;
  __syncthreads();
  const uint32_t gen = s_gen;
  const int64_t i0 = static_cast<int64_t>(c) * kArChunk + 4 * threadIdx.x;
  const bool live = i0 < a.n;  // n is a multiple of 4
  const int64_t par_off = kArDataOff + static_cast<int64_t>(gen & 1u) * a.world * a.n * 4;
  if (live) {
    const float4 v = *reinterpret_cast<const float4*>(a.in + i0);
    for (int p = 0; p < a.world; ++p)
      *reinterpret_cast<float4*>(reinterpret_cast<uint8_t*>(a.buf[p]) + par_off +
                                 (static_cast<int64_t>(a.rank) * a.n + i0) * 4) = v;
  }
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  __syncthreads();
  if (threadIdx.x < a.world) {
    uint32_t* flag = reinterpret_cast<uint32_t*>(a.buf[threadIdx.x]) + a.rank * kArMaxCtas + c;
    st_release_sys_u32(flag, gen);
  }
  if (threadIdx.x < 32) {
    bool ok = true;
    if (threadIdx.x < a.world) {
      const uint32_t* f = reinterpret_cast<const uint32_t*>(mine) + threadIdx.x * kArMaxCtas + c;
      ok = false;
      const uint32_t lim = g_wait_limit;
      for (uint32_t it = 0; it < lim; ++it) {
        if (static_cast<int32_t>(ld_acquire_sys_u32(f) - gen) >= 0) {
          ok = true;
          break;
        }
        if (it > 64) __nanosleep(32);
      }
    }
    ok = __all_sync(0xFFFFFFFFu, ok);
    if (threadIdx.x == 0) {
      s_ok = ok;
      if (!ok) atomicOr(&g_device_error, kErrWaitTimeout);
      *my_gen = gen;
    }
  }
  __syncthreads();
  if (!s_ok || !live) return;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int q = 0; q < a.world; ++q) {
    const float4 v = *reinterpret_cast<const float4*>(mine + par_off + (static_cast<int64_t>(q) * a.n + i0) * 4);
    s.x += v.x;
    s.y += v.y;
    s.z += v.z;
    s.w += v.w;
  }
  if (a.resid) {
    const float4 r = *reinterpret_cast<const float4*>(a.resid + i0);
    s.x += r.x;
    s.y += r.y;
    s.z += r.z;
    s.w += r.w;
  }
  *reinterpret_cast<float4*>(a.out + i0) = s;
}

// ---- "LL" variant: each value travels with its generation in one 8-byte word ----
// (gen << 32 | value bits), stored with 8-byte-element vector stores into slot
// [gen & 1][rank] of every rank's buffer; a receiver polls its LOCAL words until all
// carry the call's generation, so no fence and no separate flag are needed: one
// NVLink write latency per call. The data region then holds 2 x world x n 8-byte words.
__device__ __forceinline__ void st_v2u64(void* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_v2u64(const void* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__global__ void __launch_bounds__(kArThreads) allreduce_ll_kernel(const ArArgs a) {
  __shared__ uint32_t s_gen;
  __shared__ int s_ok;
  const int c = blockIdx.x;
  uint8_t* mine = reinterpret_cast<uint8_t*>(a.buf[a.rank]);
  uint32_t* my_gen = reinterpret_cast<uint32_t*>(mine + 8 * kArMaxCtas * 4) + c;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) {
    s_gen = *reinterpret_cast<volatile uint32_t*>(my_gen) + 1u;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t gen = s_gen;
  const uint64_t tag = static_cast<uint64_t>(gen) << 32;
  const int64_t i0 = static_cast<int64_t>(c) * kArChunk + 4 * threadIdx.x;
  const bool live = i0 < a.n;
  const int64_t par_off = kArDataOff + static_cast<int64_t>(gen & 1u) * a.world * a.n * 8;
  if (live) {
    const float4 v = *reinterpret_cast<const float4*>(a.in + i0);
    const uint64_t w0 = tag | __float_as_uint(v.x), w1 = tag | __float_as_uint(v.y);
    const uint64_t w2 = tag | __float_as_uint(v.z), w3 = tag | __float_as_uint(v.w);
    for (int p = 0; p < a.world; ++p) {
      uint8_t* dst = reinterpret_cast<uint8_t*>(a.buf[p]) + par_off + (static_cast<int64_t>(a.rank) * a.n + i0) * 8;
      st_v2u64(dst, w0, w1);
      st_v2u64(dst + 16, w2, w3);
    }
  }
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  bool ok = true;
  if (live) {
    const uint32_t lim = g_wait_limit;
    for (int q = 0; q < a.world && ok; ++q) {
      const uint8_t* src = mine + par_off + (static_cast<int64_t>(q) * a.n + i0) * 8;
      uint64_t w0, w1, w2, w3;
      ok = false;
      for (uint32_t it = 0; it < lim; ++it) {
        ld_v2u64(src, w0, w1);
        ld_v2u64(src + 16, w2, w3);
        if (static_cast<uint32_t>(w0 >> 32) == gen && static_cast<uint32_t>(w1 >> 32) == gen &&
            static_cast<uint32_t>(w2 >> 32) == gen && static_cast<uint32_t>(w3 >> 32) == gen) {
          ok = true;
          break;
        }
        if (it > 64) __nanosleep(32);
      }
      s.x += __uint_as_float(static_cast<uint32_t>(w0));
      s.y += __uint_as_float(static_cast<uint32_t>(w1));
      s.z += __uint_as_float(static_cast<uint32_t>(w2));
      s.w += __uint_as_float(static_cast<uint32_t>(w3));
    }
  }
  if (!ok) {
    s_ok = 0;
    atomicOr(&g_device_error, kErrWaitTimeout);
  }
  __syncthreads();
  if (threadIdx.x == 0) *my_gen = gen;
  if (!s_ok || !live) return;
  if (a.resid) {
    const float4 r = *reinterpret_cast<const float4*>(a.resid + i0);
    s.x += r.x;
    s.y += r.y;
    s.z += r.z;
    s.w += r.w;
  }
  *reinterpret_cast<float4*>(a.out + i0) = s;
}

// GGUFMM_AR_PROTO=push selects the fenced push-and-flag kernel for data calls (the
// barrier always uses it); the default is the LL kernel.
bool ar_ll() {
  static const bool on = [] {
    const char* e = std::getenv("GGUFMM_AR_PROTO");
    return !(e && e[0] == 'p');
  }();
  return on;
}

}  // namespace

size_t allreduce_buffer_bytes(int64_t n, int world) {
  if (n < 0 || n > kArMaxN || n % 4 || world < 2 || world > 8) return 0;
  return (kArDataOff + static_cast<size_t>(2) * world * n * 8 + 255) / 256 * 256;
}

cudaError_t launch_allreduce_oneshot(const float* in, float* out, int64_t n, void* const* bufs, int world, int rank,
                                     const void* resid, cudaStream_t st) {
  if (n < 0 || n > kArMaxN || n % 4 || world < 2 || world > 8 || rank < 0 || rank >= world)
    return cudaErrorInvalidValue;
  ArArgs a{};
  for (int i = 0; i < world; ++i) a.buf[i] = reinterpret_cast<uint64_t>(bufs[i]);
  a.world = world;
  a.rank = rank;
  a.n = n;
  a.in = in;
  a.out = out;
  a.resid = static_cast<const float*>(resid);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(n == 0 ? 1 : (n + kArChunk - 1) / kArChunk));
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (n > 0 && ar_ll()) return cudaLaunchKernelEx(&cfg, allreduce_ll_kernel, a);
  return cudaLaunchKernelEx(&cfg, allreduce_push_kernel, a);
}

cudaError_t allreduce_device_error(int* v, int clear, cudaStream_t st) { return tu_device_error(v, clear, st); }
cudaError_t allreduce_set_wait_limit(uint32_t polls) { return tu_set_wait_limit(polls); }

}  // namespace ggufmm
