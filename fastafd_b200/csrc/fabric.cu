// Fabric: symmetric peer-visible device buffers for one NVLink/NVSwitch domain.
//
// Each rank (one process per GPU) allocates its part of a named buffer with
// cudaMalloc, exports a CUDA IPC handle, and opens every peer's handle; the result
// is a table of base pointers, one per rank, that kernels index to store into or
// load from a peer GPU directly over NVLink. Handles travel over the host-side
// process group (gloo / TCP store) in Python. This replaces what the reference gets
// from torch symmetric memory and NCCL windows
// (python/minisgl/kernel/megamoe_m2n_mega.py:163-262,
//  python/minisgl/kernel/csrc/src/pynccl.cu:90-94).
//
// Nothing here launches work that waits on a peer; see moe_comm.cu for the bounded
// flag waits.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

extern "C" {

// Allocates `nbytes` (rounded up to 2 MiB granularity by the driver as it sees fit),
// zero-fills it, and writes a 64-byte IPC handle. Returns 0 or a cudaError_t.
int afd_fabric_alloc(size_t nbytes, void** ptr, void* handle64) {
  if (nbytes == 0) nbytes = 256;
  cudaError_t e = cudaMalloc(ptr, nbytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemset(*ptr, 0, nbytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return static_cast<int>(e);
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) return static_cast<int>(e);
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle64, &h, 64);
  return 0;
}

// Maps a peer's allocation into this process. The peer GPU must be reachable by
// P2P (NVLink); the mapping enables peer access lazily.
int afd_fabric_open(const void* handle64, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, 64);
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return static_cast<int>(e);
}

int afd_fabric_close(void* ptr) { return static_cast<int>(cudaIpcCloseMemHandle(ptr)); }

int afd_fabric_free(void* ptr) { return static_cast<int>(cudaFree(ptr)); }

// Plain device allocation without a handle (single-process runs, tests).
int afd_device_alloc(size_t nbytes, void** ptr) {
  if (nbytes == 0) nbytes = 256;
  cudaError_t e = cudaMalloc(ptr, nbytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaMemset(*ptr, 0, nbytes));
}

int afd_can_access_peer(int dev, int peer, int* out) {
  return static_cast<int>(cudaDeviceCanAccessPeer(out, dev, peer));
}

// Peer copy bandwidth probe helper: async copy between two device pointers that may
// live on different GPUs (used by the bandwidth benchmark, not by the hot path).
int afd_memcpy_async(void* dst, const void* src, size_t nbytes, void* stream) {
  return static_cast<int>(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)));
}

const char* afd_cuda_error_string(int code) { return cudaGetErrorString(static_cast<cudaError_t>(code)); }

}  // extern "C"
