// Attention tensor-parallel collectives over the fabric (peer stores + epoch flags), the
// counterparts of the NCCL calls around the TP-sharded GEMMs:
//
//   all-gather  -> qkv GEMM : tp_allgather_push_kernel stores this rank's token rows into every
//       TP peer's gather buffer (so the GEMM reads local memory only) and releases one flag per
//       peer; tp_allgather_wait_kernel orders the consumer stream after all peers' flags.
//   o_proj GEMM -> reduce-scatter : the GEMM itself pushes its partial rows from the epilogue
//       (grouped_gemm_kernel with the COMBINE epilogue and a static row map) into the owner's
//       [tp][tokens][H] buffer; ag_combine_kernel sums the tp partials after waiting for the flags.
//
// Flags carry a monotonically increasing epoch kept in device memory, so CUDA graphs replay the
// protocol. All waits are bounded and report through the status word.
// Reference: the NCCL all-reduce / all-gather around LinearOProj and the LM head,
// python/minisgl/layers/linear.py:418-447, python/minisgl/distributed/impl.py:28-85.
#include "common.cuh"

namespace afd {

constexpr int kMaxTp = 8;

struct TpGatherArgs {
  const __nv_bfloat16* x;              // [T_local][H]
  __nv_bfloat16* peer_buf[kMaxTp];     // gather buffer base in every TP rank (own rank included)
  uint32_t* peer_flag[kMaxTp];         // flag word of this source in every TP rank
  int tp, my_index, T_local, H;
  uint32_t* epoch;                     // value to publish, incremented by the last CTA
  unsigned int* done_counter;
  int* status;
};

__global__ void __launch_bounds__(256) tp_allgather_push_kernel(const TpGatherArgs a) {
  const int t = blockIdx.x;
  const __nv_bfloat16* src = a.x + static_cast<size_t>(t) * a.H;
  const size_t dst_row = static_cast<size_t>(a.my_index) * a.T_local + t;
  for (int i = threadIdx.x * 8; i < a.H; i += blockDim.x * 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + i);
    for (int p = 0; p < a.tp; ++p) *reinterpret_cast<uint4*>(a.peer_buf[p] + dst_row * a.H + i) = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // per-CTA gpu-scope fence + counter; the last CTA issues the one system-scope fence and
    // releases the flags (data -> fence.gpu -> counter -> fence.sys -> flag).
    __threadfence();
    const unsigned int prev = atomicAdd(a.done_counter, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      const uint32_t e = *a.epoch;
      for (int p = 0; p < a.tp; ++p) st_relaxed_sys(a.peer_flag[p], e);
      *a.epoch = e + 1;
      *a.done_counter = 0;
      __threadfence();
    }
  }
}

struct TpWaitArgs {
  const uint32_t* flags;   // [tp] local flag words, one per source rank
  int tp;
  uint32_t* epoch;         // expected value, incremented after the wait when `bump` is set
  uint64_t timeout_ns;
  int* status;
  int bump;
};

__global__ void tp_allgather_wait_kernel(const TpWaitArgs a) {
  // No early trigger here: the kernel behind a flag wait is a many-CTA consumer, and launched early it
  // would sit resident (registers, shared memory) for the whole wait and take SM slots from the other
  // micro-batch's attention kernel. It starts when this warp exits.
  pdl_wait();
  const uint32_t e = *a.epoch;
  if (threadIdx.x < a.tp) wait_flag_ge(a.flags + threadIdx.x, e, a.timeout_ns, a.status);
  __syncthreads();
  if (threadIdx.x == 0 && a.bump) {
    *a.epoch = e + 1;
    __threadfence();
  }
}

}  // namespace afd

struct AfdTpGatherDesc {
  const void* x;
  void* peer_buf[afd::kMaxTp];
  void* peer_flag[afd::kMaxTp];
  int tp, my_index, T_local, H;
  void* epoch; void* done_counter; void* status;
};

extern "C" int afd_tp_allgather_push(const AfdTpGatherDesc* d, void* stream) {
  using namespace afd;
  if (d->T_local == 0) return 0;
  if (d->tp < 1 || d->tp > kMaxTp || d->H % 8 != 0 || d->my_index < 0 || d->my_index >= d->tp) return -1;
  TpGatherArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(d->x);
  for (int p = 0; p < d->tp; ++p) {
    a.peer_buf[p] = static_cast<__nv_bfloat16*>(d->peer_buf[p]);
    a.peer_flag[p] = static_cast<uint32_t*>(d->peer_flag[p]);
  }
  a.tp = d->tp; a.my_index = d->my_index; a.T_local = d->T_local; a.H = d->H;
  a.epoch = static_cast<uint32_t*>(d->epoch);
  a.done_counter = static_cast<unsigned int*>(d->done_counter);
  a.status = static_cast<int*>(d->status);
  tp_allgather_push_kernel<<<d->T_local, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  AFD_CHECK_LAUNCH();
  return 0;
}

extern "C" int afd_tp_allgather_wait(const void* flags, int tp, void* epoch, unsigned long long timeout_ns,
                                     void* status, void* stream) {
  using namespace afd;
  if (tp < 1 || tp > kMaxTp) return -1;
  TpWaitArgs a{static_cast<const uint32_t*>(flags), tp, static_cast<uint32_t*>(epoch), timeout_ns,
               static_cast<int*>(status), 1};
  tp_allgather_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(a);
  AFD_CHECK_LAUNCH();
  return 0;
}

// One-warp bounded wait until `n` flag words reach the epoch stored at `epoch` (which is left
// unchanged): put in front of a many-CTA consumer so that the consumer's CTAs are not resident,
// holding shared memory and registers, while the producers are still working.
extern "C" int afd_wait_flags_epoch(const void* flags, int n, const void* epoch, unsigned long long timeout_ns,
                                    void* status, void* stream) {
  using namespace afd;
  if (n < 1 || n > 32) return -1;
  TpWaitArgs a{static_cast<const uint32_t*>(flags), n, const_cast<uint32_t*>(static_cast<const uint32_t*>(epoch)),
               timeout_ns, static_cast<int*>(status), 0};
  cudaError_t le = launch_pdl(tp_allgather_wait_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), 1, a);
  if (le != cudaSuccess) return static_cast<int>(le);
  return 0;
}
