// Entry point of the kernel library that allocates nothing.
//
// It has no counterpart in the reference project: it exists for embedders of this
// library that must not, or cannot, ask the CUDA driver for memory at call time.
// Typical cases: a serving process that has already handed every spare byte of HBM to
// its KV-cache pool, so a cudaMalloc for split-KV scratch would fail or force the pool to
// shrink; a latency-critical decode loop in which cudaMalloc / cudaFree are forbidden
// because they synchronise the whole device; and host code that runs under an allocator
// policy (a pinned arena, a sandbox) where only pre-registered memory may be touched.
//
// The split-KV partial results of the paged decode attention kernel normally live in a
// caller-provided workspace. This variant keeps them in a fixed array that is part of
// the library image itself, so every GPU that loads the library carries
// AFD_NOALLOC_SCRATCH_BYTES of it until the process exits.
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

// Size of the built-in scratch array (8 MiB). A call whose split-KV partials need more
// is rejected with AFD_NOALLOC_ERR_TOO_LARGE; nothing is launched in that case.
#define AFD_NOALLOC_SCRATCH_BYTES (8u * 1024u * 1024u)

#define AFD_NOALLOC_ERR_TOO_LARGE (-20)   // scratch need exceeds AFD_NOALLOC_SCRATCH_BYTES
#define AFD_NOALLOC_ERR_DEVICE (-21)      // current device index outside the supported range

// Paged GQA decode attention with split KV, same contract as afd_decode_attention
// (q [B*q_len][Hq][D] bf16, k/v caches [slots][Hkv][D] bf16, page_table [B][max_pages]
// int32, seq_lens [B] int32, out like q) except that no workspace is passed.
//
// * Calls no cudaMalloc / cudaFree / allocating library routine. The caller still owns and
//   passes all inputs and the output.
// * The first call on each device resolves the device address of the built-in array
//   (cudaGetSymbolAddress, with that device current). Make that first call outside of any
//   stream capture.
// * All calls on a device share the one array and it keeps whatever the previous call left
//   there. Two things live in it. The per-tile arrival counters occupy a fixed region at the
//   front of the array, whatever B and splits are; they start at zero (the array is
//   zero-initialised when the library is loaded) and every finished call leaves them at zero,
//   so the next call, of any shape, finds them clear. The partial results behind them are
//   written by a call before that call reads them, so their leftovers need no clearing.
//   A call that was cut short (its status word reports a timeout) can leave counters non-zero:
//   do not reuse the entry point on that device after such a failure.
// * Two calls whose kernels overlap in time on the same GPU (different streams) race on the
//   array: serialise them.
// Returns 0, a positive cudaError_t, or a negative argument error (see
// afd_noalloc_strerror).
int afd_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                 const void* page_table, const void* seq_lens, void* out, int B,
                                 int Hq, int Hkv, int D, int q_len, int page_size, int max_pages,
                                 long cache_slots, int splits, float sm_scale, void* status,
                                 void* stream);

// Bytes of scratch a call with these sizes needs (compare with AFD_NOALLOC_SCRATCH_BYTES).
long afd_decode_attention_noalloc_need(int B, int Hq, int Hkv, int q_len, int D, int splits);

// Human-readable text for a negative return code of the entry point above.
const char* afd_noalloc_strerror(int code);

#ifdef __cplusplus
}
#endif
