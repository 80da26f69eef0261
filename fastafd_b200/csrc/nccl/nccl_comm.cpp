// Thin NCCL communicator for the attention-side tensor-parallel collectives.
//
// One communicator per TP group, created from a unique id that rank 0 of the group shares
// over the host-side process group. Small all-reduces go through a persistent buffer that
// is allocated with ncclMemAlloc and registered with the communicator, so that NCCL can use
// its NVLink SHARP (NVLS) path on an NVSwitch machine without per-call registration; large
// ones run in place. Errors are polled (ncclCommGetAsyncError) and a communicator can be
// aborted from the host, which is how a hung collective is abandoned after a peer died.
//
// Reference: python/minisgl/kernel/csrc/src/pynccl.cu (NCCLWrapper: init :80, symmetric
// buffer :90-94, all_reduce :121-134, all_gather :170, get_async_error :183, abort :197).
#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>
#include <string.h>

#include <new>

struct AfdNcclComm {
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  void* buf = nullptr;        // registered staging buffer
  void* reg = nullptr;        // registration handle
  size_t buf_bytes = 0;
};

static ncclDataType_t to_nccl(int dtype) {
  switch (dtype) {
    case 0: return ncclBfloat16;
    case 1: return ncclFloat32;
    case 2: return ncclFloat16;
    case 3: return ncclInt32;
    default: return ncclUint8;
  }
}
static size_t elem_size(int dtype) { return dtype == 1 || dtype == 3 ? 4 : (dtype == 4 ? 1 : 2); }

extern "C" {

int afd_nccl_unique_id(void* out128) {
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return static_cast<int>(r);
  static_assert(sizeof(id) == 128, "unique id size");
  memcpy(out128, &id, 128);
  return 0;
}

// max_buffer_bytes = 0 disables the staging buffer (every collective runs in place).
int afd_nccl_init(int rank, int world, const void* id128, size_t max_buffer_bytes, void** handle) {
  AfdNcclComm* c = new (std::nothrow) AfdNcclComm();
  if (c == nullptr) return -1;
  ncclUniqueId id;
  memcpy(&id, id128, 128);
  ncclResult_t r = ncclCommInitRank(&c->comm, world, id, rank);
  if (r != ncclSuccess) {
    delete c;
    return static_cast<int>(r);
  }
  c->rank = rank;
  c->world = world;
  if (max_buffer_bytes > 0) {
    if (ncclMemAlloc(&c->buf, max_buffer_bytes) == ncclSuccess) {
      c->buf_bytes = max_buffer_bytes;
      if (ncclCommRegister(c->comm, c->buf, max_buffer_bytes, &c->reg) != ncclSuccess) c->reg = nullptr;
    } else {
      c->buf = nullptr;
    }
  }
  *handle = c;
  return 0;
}

int afd_nccl_all_reduce(void* handle, void* data, size_t count, int dtype, void* stream) {
  AfdNcclComm* c = static_cast<AfdNcclComm*>(handle);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t bytes = count * elem_size(dtype);
  if (c->buf != nullptr && bytes <= c->buf_bytes) {
    cudaError_t e = cudaMemcpyAsync(c->buf, data, bytes, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return 1000 + static_cast<int>(e);
    ncclResult_t r = ncclAllReduce(c->buf, c->buf, count, to_nccl(dtype), ncclSum, c->comm, st);
    if (r != ncclSuccess) return static_cast<int>(r);
    e = cudaMemcpyAsync(data, c->buf, bytes, cudaMemcpyDeviceToDevice, st);
    return e == cudaSuccess ? 0 : 1000 + static_cast<int>(e);
  }
  return static_cast<int>(ncclAllReduce(data, data, count, to_nccl(dtype), ncclSum, c->comm, st));
}

// recv holds world * count elements; rank r's contribution lands at recv + r * count.
int afd_nccl_all_gather(void* handle, const void* send, void* recv, size_t count, int dtype, void* stream) {
  AfdNcclComm* c = static_cast<AfdNcclComm*>(handle);
  return static_cast<int>(ncclAllGather(send, recv, count, to_nccl(dtype), c->comm, static_cast<cudaStream_t>(stream)));
}

// send holds world * count elements; recv gets the sum of every rank's r-th block.
int afd_nccl_reduce_scatter(void* handle, const void* send, void* recv, size_t count, int dtype, void* stream) {
  AfdNcclComm* c = static_cast<AfdNcclComm*>(handle);
  return static_cast<int>(ncclReduceScatter(send, recv, count, to_nccl(dtype), ncclSum, c->comm,
                                            static_cast<cudaStream_t>(stream)));
}

int afd_nccl_async_error(void* handle, int* out) {
  AfdNcclComm* c = static_cast<AfdNcclComm*>(handle);
  ncclResult_t state = ncclSuccess;
  ncclResult_t r = ncclCommGetAsyncError(c->comm, &state);
  *out = static_cast<int>(state);
  return static_cast<int>(r);
}

int afd_nccl_abort(void* handle) {
  AfdNcclComm* c = static_cast<AfdNcclComm*>(handle);
  if (c->comm == nullptr) return 0;
  ncclResult_t r = ncclCommAbort(c->comm);
  c->comm = nullptr;
  return static_cast<int>(r);
}

int afd_nccl_destroy(void* handle) {
  AfdNcclComm* c = static_cast<AfdNcclComm*>(handle);
  if (c->comm != nullptr) {
    if (c->reg != nullptr) ncclCommDeregister(c->comm, c->reg);
    if (c->buf != nullptr) ncclMemFree(c->buf);
    ncclCommDestroy(c->comm);
  }
  delete c;
  return 0;
}

const char* afd_nccl_error_string(int code) { return ncclGetErrorString(static_cast<ncclResult_t>(code)); }

}  // extern "C"
