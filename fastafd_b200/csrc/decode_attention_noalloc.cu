// Allocation-free variant of the paged decode attention entry point: the split-KV
// partials go to a file-scope device array instead of a caller workspace. See
// fastafd_noalloc.h for who needs this and for the rules of use.
#include "fastafd_noalloc.h"

#include <cuda_runtime.h>
#include <mutex>

extern "C" long afd_decode_attn_workspace_bytes(int B, int Hq, int Hkv, int q_len, int D, int splits);
extern "C" int afd_decode_attention(const void* q, const void* k_cache, const void* v_cache,
                                    const void* page_table, const void* seq_lens, void* out,
                                    void* workspace, int B, int Hq, int Hkv, int D, int q_len,
                                    int page_size, int max_pages, long cache_slots, int splits,
                                    float sm_scale, void* status, void* stream);

namespace {

// The scratch itself. In host code this name is only a stand-in for the symbol; the device
// address comes from cudaGetSymbolAddress below and is what the kernel receives.
static __device__ __align__(256) unsigned char g_noalloc_scratch[AFD_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void* g_scratch_addr[kMaxDevices] = {};
std::once_flag g_once[kMaxDevices];
cudaError_t g_setup_err[kMaxDevices] = {};

// Once per device, with that device current.
cudaError_t scratch_for_current_device(int dev, void** out) {
  std::call_once(g_once[dev], [dev]() {
    void* p = nullptr;
    g_setup_err[dev] = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    g_scratch_addr[dev] = p;
  });
  *out = g_scratch_addr[dev];
  return g_setup_err[dev];
}

}  // namespace

extern "C" long afd_decode_attention_noalloc_need(int B, int Hq, int Hkv, int q_len, int D, int splits) {
  return splits > 1 ? afd_decode_attn_workspace_bytes(B, Hq, Hkv, q_len, D, splits) : 0;
}

extern "C" const char* afd_noalloc_strerror(int code) {
  switch (code) {
    case 0: return "ok";
    case AFD_NOALLOC_ERR_TOO_LARGE:
      return "split-KV partials need more than the built-in scratch array "
             "(AFD_NOALLOC_SCRATCH_BYTES); use fewer splits or a smaller batch, or call "
             "afd_decode_attention with your own workspace";
    case AFD_NOALLOC_ERR_DEVICE: return "current CUDA device index is outside the supported range";
    default: return "invalid arguments (same codes as afd_decode_attention)";
  }
}

extern "C" int afd_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                            const void* page_table, const void* seq_lens, void* out,
                                            int B, int Hq, int Hkv, int D, int q_len, int page_size,
                                            int max_pages, long cache_slots, int splits, float sm_scale,
                                            void* status, void* stream) {
  if (Hkv <= 0 || Hq % Hkv != 0 || splits < 1) return -1;
  const long need = afd_decode_attention_noalloc_need(B, Hq, Hkv, q_len, D, splits);
  if (need > static_cast<long>(AFD_NOALLOC_SCRATCH_BYTES)) return AFD_NOALLOC_ERR_TOO_LARGE;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= kMaxDevices) return AFD_NOALLOC_ERR_DEVICE;
  void* scratch = nullptr;
  e = scratch_for_current_device(dev, &scratch);
  if (e != cudaSuccess) return static_cast<int>(e);
  return afd_decode_attention(q, k_cache, v_cache, page_table, seq_lens, out, scratch, B, Hq, Hkv, D,
                              q_len, page_size, max_pages, cache_slots, splits, sm_scale, status, stream);
}
