// Token sampling: temperature softmax, top-k and top-p filtering and one multinomial draw per
// row, in one launch (one CTA per row). Rows with temperature <= 0 take the arg-max (lowest
// index among equals).
//
// The filters are thresholds on the probability: top-k keeps p >= (k-th largest p); top-p keeps
// a token when the mass of the strictly larger probabilities (after the top-k filter, not
// renormalised) is <= top_p. Both thresholds are found by a 4-level radix select over the bits
// of p (8 bits per level; histograms of count and mass in shared memory), the two selects share
// their passes over the row. The draw is an inverse CDF over the kept tokens in index order
// from a caller-supplied uniform number, so the host owns the random stream.
//
// The reference samples with FlashInfer (softmax + top_k_top_p_sampling_from_probs,
// python/minisgl/engine/sample.py:19-75); the filter semantics follow that path.
#include "common.cuh"

namespace afd {

namespace {

constexpr int kSampleThreads = 1024;
constexpr int kBins = 256;

template <typename T>
__device__ __forceinline__ float load_logit(const T* p, int i);
template <>
__device__ __forceinline__ float load_logit<float>(const float* p, int i) { return p[i]; }
template <>
__device__ __forceinline__ float load_logit<__nv_bfloat16>(const __nv_bfloat16* p, int i) {
  return __bfloat162float(p[i]);
}

__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < (blockDim.x >> 5) ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

}  // namespace

template <typename T>
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(
    const T* __restrict__ logits, long ld, int V, const float* __restrict__ temperatures,
    const int* __restrict__ top_ks, const float* __restrict__ top_ps, const float* __restrict__ uniform,
    int* __restrict__ out) {
  const int row = blockIdx.x;
  const T* x = logits + static_cast<size_t>(row) * ld;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __shared__ float red[32];
  __shared__ int red_i[32];
  __shared__ unsigned int h_cnt[2][kBins];
  __shared__ float h_mass[2][kBins];
  __shared__ unsigned int s_prefix[2];
  __shared__ float s_carry_mass;          // top-p: mass strictly above the current prefix
  __shared__ unsigned int s_carry_cnt;    // top-k: count strictly above the current prefix
  __shared__ float s_scan[kSampleThreads / 32];
  __shared__ int s_pick;

  // ---- pass 1: max and arg-max ----
  float mx = -INFINITY;
  int mi = 0x7fffffff;
  for (int i = tid; i < V; i += kSampleThreads) {
    const float v = load_logit(x, i);
    if (v > mx) {            // strictly greater keeps the lowest index of this thread's stride
      mx = v;
      mi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, mx, o);
    const int oi = __shfl_xor_sync(0xffffffffu, mi, o);
    if (ov > mx || (ov == mx && oi < mi)) {
      mx = ov;
      mi = oi;
    }
  }
  if (lane == 0) {
    red[warp] = mx;
    red_i[warp] = mi;
  }
  __syncthreads();
  mx = red[0];
  mi = red_i[0];
  for (int w = 1; w < kSampleThreads / 32; ++w) {
    if (red[w] > mx || (red[w] == mx && red_i[w] < mi)) {
      mx = red[w];
      mi = red_i[w];
    }
  }
  const float temp = temperatures[row];
  if (!(temp > 0.f)) {
    if (tid == 0) out[row] = mi;
    return;
  }
  const float inv_t = 1.f / temp;

  // ---- pass 2: partition function ----
  float z = 0.f;
  for (int i = tid; i < V; i += kSampleThreads) z += __expf((load_logit(x, i) - mx) * inv_t);
  z = block_reduce_sum(z, red);
  const float inv_z = 1.f / z;

  int k = top_ks[row];
  if (k <= 0 || k > V) k = V;
  const float tp = top_ps[row];
  const bool need_k = k < V, need_p = tp < 1.f;

  // ---- radix select of both thresholds (keys = bits of p, monotone for p >= 0) ----
  unsigned int thr_k = 0u, thr_p = 0u;     // keep p with bits >= threshold
  if (need_k || need_p) {
    if (tid == 0) {
      s_prefix[0] = s_prefix[1] = 0u;
      s_carry_mass = 0.f;
      s_carry_cnt = 0u;
    }
    // top-p runs on the top-k-filtered distribution, so the k-threshold is found first.
    for (int sel = need_k ? 0 : 1; sel < (need_p ? 2 : 1); ++sel) {
      if (tid == 0) {
        s_carry_mass = 0.f;
        s_carry_cnt = 0u;
      }
      for (int level = 3; level >= 0; --level) {
        for (int b = tid; b < kBins; b += kSampleThreads) {
          h_cnt[sel][b] = 0u;
          h_mass[sel][b] = 0.f;
        }
        __syncthreads();
        const unsigned int prefix = s_prefix[sel];
        const int shift = level * 8;
        const unsigned int hi_mask = level == 3 ? 0u : (0xffffffffu << (shift + 8));
        for (int i = tid; i < V; i += kSampleThreads) {
          const float p = __expf((load_logit(x, i) - mx) * inv_t) * inv_z;
          const unsigned int key = __float_as_uint(p);
          if (sel == 1 && key < thr_k) continue;                 // removed by top-k
          if ((key & hi_mask) != (prefix & hi_mask)) continue;   // not under the current prefix
          const unsigned int bin = (key >> shift) & 0xffu;
          atomicAdd(&h_cnt[sel][bin], 1u);
          if (sel == 1) atomicAdd(&h_mass[sel][bin], p);
        }
        __syncthreads();
        if (tid == 0) {
          int chosen = 0;
          if (sel == 0) {
            // highest bin at which the count from above reaches k
            unsigned int above = s_carry_cnt;
            for (int b = kBins - 1; b >= 0; --b) {
              if (above + h_cnt[0][b] >= static_cast<unsigned int>(k)) {
                chosen = b;
                break;
              }
              above += h_cnt[0][b];
            }
            s_carry_cnt = above;
          } else {
            // lowest non-empty bin whose strictly-larger mass is still <= top_p
            float above = s_carry_mass;
            chosen = -1;
            for (int b = kBins - 1; b >= 0; --b) {
              if (h_cnt[1][b] == 0u) continue;
              if (above <= tp || chosen < 0) chosen = b;          // the largest token is always kept
              else break;
              if (above + h_mass[1][b] > tp) break;               // nothing below this bin survives
              above += h_mass[1][b];
            }
            if (chosen < 0) chosen = 0;
            // mass strictly above the chosen bin
            float m = s_carry_mass;
            for (int b = kBins - 1; b > chosen; --b) m += h_mass[1][b];
            s_carry_mass = m;
          }
          s_prefix[sel] = prefix | (static_cast<unsigned int>(chosen) << shift);
        }
        __syncthreads();
      }
      if (sel == 0) thr_k = s_prefix[0];
      else thr_p = s_prefix[1];
      __syncthreads();
    }
  }
  const unsigned int thr = thr_k > thr_p ? thr_k : thr_p;

  // ---- kept mass per thread over a contiguous chunk, block scan, inverse CDF ----
  const int chunk = (V + kSampleThreads - 1) / kSampleThreads;
  const int lo = tid * chunk, hi = min(V, lo + chunk);
  float mine = 0.f;
  for (int i = lo; i < hi; ++i) {
    const float p = __expf((load_logit(x, i) - mx) * inv_t) * inv_z;
    if (__float_as_uint(p) >= thr) mine += p;
  }
  // inclusive scan over threads
  float incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) s_scan[warp] = incl;
  if (tid == 0) s_pick = -1;
  __syncthreads();
  if (warp == 0) {
    float w = s_scan[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    s_scan[lane] = w;
  }
  __syncthreads();
  const float before_warp = warp == 0 ? 0.f : s_scan[warp - 1];
  const float total = s_scan[kSampleThreads / 32 - 1];
  const float end = before_warp + incl, begin = end - mine;
  const float target = fminf(fmaxf(uniform[row], 0.f), 0.99999994f) * total;
  if (mine > 0.f && target >= begin && target < end) {
    float run = begin;
    int pick = -1;
    for (int i = lo; i < hi; ++i) {
      const float p = __expf((load_logit(x, i) - mx) * inv_t) * inv_z;
      if (__float_as_uint(p) >= thr) {
        pick = i;
        run += p;
        if (run > target) break;
      }
    }
    if (pick >= 0) atomicMax(&s_pick, pick);
  }
  __syncthreads();
  if (tid == 0) out[row] = s_pick >= 0 ? s_pick : mi;   // rounding at a chunk border: fall back to the mode
}

}  // namespace afd

// logits [T][ld] (bf16 or fp32, V valid columns; ld 0 broadcasts one row); temperatures / top_ps / uniform fp32 [T];
// top_ks int32 [T] (<= 0: off); out int32 [T].
extern "C" int afd_sample(const void* logits, long ld, int T, int V, int is_bf16, const void* temperatures,
                          const void* top_ks, const void* top_ps, const void* uniform, void* out,
                          void* stream) {
  using namespace afd;
  if (T == 0) return 0;
  if (V <= 0 || (ld < V && ld != 0)) return -1;   // ld == 0: every row reads the same logits
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (is_bf16) {
    sample_kernel<__nv_bfloat16><<<T, kSampleThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(logits), ld, V, static_cast<const float*>(temperatures),
        static_cast<const int*>(top_ks), static_cast<const float*>(top_ps), static_cast<const float*>(uniform),
        static_cast<int*>(out));
  } else {
    sample_kernel<float><<<T, kSampleThreads, 0, st>>>(
        static_cast<const float*>(logits), ld, V, static_cast<const float*>(temperatures),
        static_cast<const int*>(top_ks), static_cast<const float*>(top_ps), static_cast<const float*>(uniform),
        static_cast<int*>(out));
  }
  AFD_CHECK_LAUNCH();
  return 0;
}
