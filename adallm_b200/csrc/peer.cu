// Peer memory for tensor parallelism over NVLink (one process per GPU).
//
// The row-parallel projections of a decoder layer (o_proj, down_proj; the reference
// all-reduces their outputs with NCCL, adallm/ops/linear.py:193-215) write their split-K
// partial planes straight into every rank's inbox through CUDA IPC mappings of the peers'
// buffers, each fp32 value with the step's tag in the same 8-byte store; the consumer on each
// rank (RMSNorm + quantise) polls the words until their tags are current and sums the planes
// of all ranks in rank order, so every rank computes the same residual stream.  A
// system-scope release (fence + counter) costs 4.5-15 us per GEMM on B200, the tagged words
// nothing beyond the doubled bytes.  These entry points set the buffers up; the data path
// lives in the GEMM epilogue (nvfp4_gemm.cu) and the RMSNorm producer (fused.cu).  Plain peer
// stores and loads only: no NVLink multicast object, no TMA from peer memory.
#include <cstring>

#include "common.cuh"

namespace ada {
namespace peer {

// Advance the step epoch after the last consumer of the step (programmatic launch: waits for it).
__global__ void epoch_advance_kernel(uint32_t* epoch) {
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) *epoch += 1u;
}

}  // namespace peer
}  // namespace ada

using namespace ada;

extern "C" int ada_peer_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return ADA_ERR_INVALID_ARG;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return ADA_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return ADA_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == ADA_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return ADA_OK;
}

extern "C" int ada_peer_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return ADA_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? ADA_OK : ADA_ERR_CUDA;
}

extern "C" int ada_peer_close(void* ptr) {
  if (!ptr) return ADA_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? ADA_OK : ADA_ERR_CUDA;
}

extern "C" int ada_peer_free(void* ptr) {
  if (!ptr) return ADA_ERR_INVALID_ARG;
  return cudaFree(ptr) == cudaSuccess ? ADA_OK : ADA_ERR_CUDA;
}

extern "C" int ada_tp_epoch_advance(uint32_t* epoch, void* stream) {
  if (!epoch) return ADA_ERR_INVALID_ARG;
  (void)launch_k(peer::epoch_advance_kernel, dim3(1), dim3(32), 0, reinterpret_cast<cudaStream_t>(stream), epoch);
  ADA_CHECK_LAUNCH();
  return ADA_OK;
}
