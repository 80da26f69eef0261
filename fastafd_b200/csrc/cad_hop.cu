// Hop kernels of core-attention disaggregation (CAD): the model GPU keeps everything except the KV
// cache and the decode attention core, which live on attention GPUs. Per layer and micro-batch the
// model GPU puts the q|k|v rows of the requests an attention GPU owns into that GPU's window and
// releases a flag; the attention GPU waits for it, stores K/V into its paged pool, runs attention with
// the output written straight into the model GPU's window, and releases the o flag.
//
//   cad_put_rows_kernel    selected rows -> peer window slot (rows compacted), last CTA releases
//                          flag = epoch + 1
//   cad_wait_store_kernel  bounded wait for the qkv flag, then K/V rows of the window into the pool
//   cad_wait_kernel        bounded wait for n flags (the o flags of the attention GPUs)
//   cad_flag_kernel        system fence + release flag = epoch + 1 (after a kernel that wrote peer memory)
//   cad_epoch_kernel       epoch += 1, the last kernel of a step
//
// Flags are stamped with the step's epoch, so they are never reset; every wait is bounded, records
// a code in the window's err word when it gives up, and returns at once when the word is already set.
// Reference: python/minisgl/kernel/cad_hop.py:42-204, python/minisgl/cad/model_side.py:117-130,
// python/minisgl/cad/attn_side.py:178-191.
#include "common.cuh"

namespace afd {

struct CadPutArgs {
  const __nv_bfloat16* src;   // [T][src_ld]
  long src_ld;
  const int* sel;             // [n] source row of every destination row (null: identity)
  int n, row_elems;
  __nv_bfloat16* dst;         // peer slot [n][row_elems]
  uint32_t* peer_flag;
  const uint32_t* epoch;
  unsigned int* done_counter;
};

__global__ void __launch_bounds__(256) cad_put_rows_kernel(const CadPutArgs a) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x;
  if (i < a.n) {
    const int r = a.sel ? a.sel[i] : i;
    const uint4* s = reinterpret_cast<const uint4*>(a.src + static_cast<size_t>(r) * a.src_ld);
    uint4* d = reinterpret_cast<uint4*>(a.dst + static_cast<size_t>(i) * a.row_elems);
    for (int v = threadIdx.x; v < a.row_elems / 8; v += blockDim.x) d[v] = s[v];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(a.done_counter, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      st_relaxed_sys(a.peer_flag, *a.epoch + 1u);
      *a.done_counter = 0;
      __threadfence();
    }
  }
}

struct CadWaitStoreArgs {
  const uint32_t* flag;
  const uint32_t* epoch;
  const __nv_bfloat16* rows;  // window slot [n][row_elems]: q | k | v per row
  const int* out_loc;         // [n] cache slot of each row (-1: skip)
  __nv_bfloat16* k_cache;     // [slots][Hkv][D]
  __nv_bfloat16* v_cache;
  int n, row_elems, q_elems, kv_elems;
  long cache_slots;
  uint64_t timeout_ns;
  int* err;
};

__global__ void __launch_bounds__(128) cad_wait_store_kernel(const CadWaitStoreArgs a) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) wait_flag_ge(a.flag, *a.epoch + 1u, a.timeout_ns, a.err);
  __syncthreads();
  if (*reinterpret_cast<volatile int*>(a.err) != 0) return;
  const int i = blockIdx.x;
  if (i >= a.n) return;
  const long slot = a.out_loc[i];
  if (slot < 0 || slot >= a.cache_slots) {
    if (slot != -1 && threadIdx.x == 0) set_status(a.err, kStatusBadExtent);
    return;
  }
  const uint4* k = reinterpret_cast<const uint4*>(a.rows + static_cast<size_t>(i) * a.row_elems + a.q_elems);
  const uint4* v = reinterpret_cast<const uint4*>(a.rows + static_cast<size_t>(i) * a.row_elems + a.q_elems + a.kv_elems);
  uint4* kd = reinterpret_cast<uint4*>(a.k_cache + static_cast<size_t>(slot) * a.kv_elems);
  uint4* vd = reinterpret_cast<uint4*>(a.v_cache + static_cast<size_t>(slot) * a.kv_elems);
  for (int x = threadIdx.x; x < a.kv_elems / 8; x += blockDim.x) {
    kd[x] = k[x];
    vd[x] = v[x];
  }
}

__global__ void cad_wait_kernel(const uint32_t* flags, long flag_stride, int n, const uint32_t* epoch,
                                uint64_t timeout_ns, int* err) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x < n) wait_flag_ge(flags + static_cast<size_t>(threadIdx.x) * flag_stride, *epoch + 1u, timeout_ns, err);
}

__global__ void cad_flag_kernel(uint32_t* peer_flag, const uint32_t* epoch) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(peer_flag, *epoch + 1u);
  }
}

__global__ void cad_epoch_kernel(uint32_t* epoch) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) *epoch += 1u;
}

}  // namespace afd

using namespace afd;

extern "C" int afd_cad_put_rows(const void* src, long src_ld, const void* sel, int n, int row_elems, void* dst,
                                void* peer_flag, const void* epoch, void* done_counter, void* stream) {
  if (row_elems % 8 != 0 || src_ld % 8 != 0 || n < 0) return -1;
  CadPutArgs a{static_cast<const __nv_bfloat16*>(src), src_ld, static_cast<const int*>(sel), n, row_elems,
               static_cast<__nv_bfloat16*>(dst), static_cast<uint32_t*>(peer_flag), static_cast<const uint32_t*>(epoch),
               static_cast<unsigned int*>(done_counter)};
  cudaError_t e = launch_pdl(cad_put_rows_kernel, dim3(n > 0 ? n : 1), dim3(256), 0, static_cast<cudaStream_t>(stream), 1, a);
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int afd_cad_wait_store(const void* flag, const void* epoch, const void* rows, const void* out_loc, void* k_cache,
                                  void* v_cache, int n, int row_elems, int q_elems, int kv_elems, long cache_slots,
                                  unsigned long long timeout_ns, void* err, void* stream) {
  if (row_elems % 8 != 0 || q_elems % 8 != 0 || kv_elems % 8 != 0 || q_elems + 2 * kv_elems != row_elems || err == nullptr) return -1;
  CadWaitStoreArgs a{static_cast<const uint32_t*>(flag), static_cast<const uint32_t*>(epoch),
                     static_cast<const __nv_bfloat16*>(rows), static_cast<const int*>(out_loc),
                     static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), n, row_elems, q_elems,
                     kv_elems, cache_slots, timeout_ns, static_cast<int*>(err)};
  cudaError_t e = launch_pdl(cad_wait_store_kernel, dim3(n > 0 ? n : 1), dim3(128), 0, static_cast<cudaStream_t>(stream), 1, a);
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int afd_cad_wait(const void* flags, long flag_stride, int n, const void* epoch, unsigned long long timeout_ns,
                            void* err, void* stream) {
  if (n < 1 || n > 32) return -1;
  cudaError_t e = launch_pdl(cad_wait_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), 1,
                             static_cast<const uint32_t*>(flags), flag_stride, n, static_cast<const uint32_t*>(epoch),
                             static_cast<uint64_t>(timeout_ns), static_cast<int*>(err));
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int afd_cad_flag(void* peer_flag, const void* epoch, void* stream) {
  cudaError_t e = launch_pdl(cad_flag_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), 1,
                             static_cast<uint32_t*>(peer_flag), static_cast<const uint32_t*>(epoch));
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}

extern "C" int afd_cad_epoch(void* epoch, void* stream) {
  cudaError_t e = launch_pdl(cad_epoch_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), 1,
                             static_cast<uint32_t*>(epoch));
  return e == cudaSuccess ? 0 : static_cast<int>(e);
}
