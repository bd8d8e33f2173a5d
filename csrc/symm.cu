// Symmetric device buffers for in-kernel collectives over NVLink.
// Reference counterpart: the TP all-reduce after row-parallel projections, an NCCL call
// (src/graspo/backends/graspoflow/tensor_utils.py:146-164).
//
// Every rank of a tensor-parallel group allocates a buffer of the same size
// with cudaMalloc, exports a CUDA IPC handle, and opens the handles of its
// peers (cudaIpcOpenMemHandle with lazy peer access), so a kernel on one GPU
// can store into, and atomically signal, a peer's buffer directly: the
// fused GEMM + all-reduce of the decode loop pushes each finished output tile
// into the peers' receive slots and bumps their arrival counters, and the
// consumer kernel waits for the arrivals (bounded) and sums the slots in rank
// order, so every rank computes bit-identical results.
//
// The handle exchange itself is host-side (torch.distributed, see
// graspo_b200/parallel/symm.py).

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <cstring>
#include <vector>

namespace gb {

// Allocate `nbytes` (zero-filled) and return {buffer (uint8, on the device),
// IPC handle (uint8, CPU)}.  The buffer is freed when the tensor dies.
std::vector<torch::Tensor> symm_alloc(int64_t nbytes, int64_t device) {
  TORCH_CHECK(nbytes > 0, "symmetric buffer size must be positive");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, static_cast<size_t>(nbytes)));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, static_cast<size_t>(nbytes)));
  cudaIpcMemHandle_t handle;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&handle, ptr));
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, device);
  torch::Tensor buf = torch::from_blob(
      ptr, {nbytes}, [device](void* p) {
        const c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
        cudaFree(p);
      },
      opts);
  torch::Tensor h = torch::empty({static_cast<int64_t>(sizeof(handle))}, torch::kUInt8);
  std::memcpy(h.data_ptr(), &handle, sizeof(handle));
  return {buf, h};
}

// Map a peer's buffer into this process; returns its device address.
int64_t symm_open(torch::Tensor handle, int64_t device) {
  TORCH_CHECK(handle.numel() == static_cast<int64_t>(sizeof(cudaIpcMemHandle_t)) && handle.device().is_cpu(),
              "expected a CPU uint8 IPC handle");
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.contiguous().data_ptr(), sizeof(h));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

// Let kernels on `device` read and write `peer`'s memory directly (one process
// driving several GPUs: profiling and single-process tests of the peer paths).
// Returns false when the two devices cannot reach each other.
bool enable_peer_access(int64_t device, int64_t peer) {
  int ok = 0;
  C10_CUDA_CHECK(cudaDeviceCanAccessPeer(&ok, static_cast<int>(device), static_cast<int>(peer)));
  if (!ok) return false;
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  const cudaError_t e = cudaDeviceEnablePeerAccess(static_cast<int>(peer), 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    (void)cudaGetLastError();
    return true;
  }
  C10_CUDA_CHECK(e);
  return true;
}

void symm_close(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

}  // namespace gb
