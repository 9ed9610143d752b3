// stage.cu -- ggufmm_stage_copy: host <-> device staging of a decode step's
// activations and outputs by a kernel, in place of a copy-engine memcpy.
//
// The reference moves data between host and GPU through WebGPU buffers:
// create_buffer_with_data for uploads and a staging buffer mapped for readback
// (vllm_webgpu/webgpu/buffer.py:34, :46-63). Here a decode step is one CUDA-graph
// replay, and each host <-> device copy in it was a memcpy node: the copy engine
// and the kernels hand over to each other around every such node. A kernel that
// reads (or writes) page-locked host memory directly over the bus keeps the whole
// step on the SMs and chains with the projections by programmatic dependent
// launch: the first GEMV streams its weights while this kernel is still pulling
// the activations in.
//
// The host buffer must be page-locked and mapped for the device (memory from
// cudaHostAlloc / torch's pin_memory on a system with unified addressing); its
// device address comes from cudaHostGetDevicePointer.
#include <algorithm>

#include "common.cuh"

namespace ggufmm {

int record_cuda_status(cudaError_t e);  // capi.cu: keeps the code for ggufmm_last_cuda_error

namespace {

// n16 16-byte words then `tail` (< 16) bytes; one word per thread per step.
__global__ void __launch_bounds__(256) stage_copy_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src,
                                                         int64_t n16, int tail) {
  pdl_wait();  // src may be written, dst still read, by the previous kernel
  pdl_trigger();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n16; i += stride)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  if (blockIdx.x == 0 && static_cast<int>(threadIdx.x) < tail) dst[n16 * 16 + threadIdx.x] = src[n16 * 16 + threadIdx.x];
}

// Device-side address of p: itself for device memory, the mapped address for
// page-locked host memory; null for pageable host memory.
cudaError_t device_view(const void* p, void** out) {
  cudaPointerAttributes at;
  cudaError_t e = cudaPointerGetAttributes(&at, p);
  if (e != cudaSuccess) return e;
  if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) {
    *out = const_cast<void*>(p);
    return cudaSuccess;
  }
  if (at.type != cudaMemoryTypeHost) {
    *out = nullptr;
    return cudaSuccess;
  }
  return cudaHostGetDevicePointer(out, const_cast<void*>(p), 0);
}

}  // namespace

}  // namespace ggufmm

using namespace ggufmm;

extern "C" int ggufmm_stage_copy(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return GGUFMM_OK;
  if (!dst || !src) return GGUFMM_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(dst) & 15) || (reinterpret_cast<uintptr_t>(src) & 15)) return GGUFMM_ERR_ALIGN;
  void* d = nullptr;
  void* s = nullptr;
  cudaError_t e = device_view(dst, &d);
  if (e == cudaSuccess) e = device_view(src, &s);
  if (e != cudaSuccess) {
    cudaGetLastError();  // a failed pointer query is not sticky: clear it
    return record_cuda_status(e);
  }
  if (!d || !s) return GGUFMM_ERR_ARG;  // pageable host memory: not reachable by a kernel
  if ((reinterpret_cast<uintptr_t>(d) & 15) || (reinterpret_cast<uintptr_t>(s) & 15)) return GGUFMM_ERR_ALIGN;
  const int64_t n16 = static_cast<int64_t>(bytes / 16);
  const int tail = static_cast<int>(bytes % 16);
  // one 16-byte request per thread: as many in flight as possible to cover the bus latency
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((n16 + 255) / 256, 1024));
  e = pdl_launch(stage_copy_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                 static_cast<cudaStream_t>(stream), static_cast<uint8_t*>(d), static_cast<const uint8_t*>(s), n16,
                 tail);
  return record_cuda_status(e);
}
