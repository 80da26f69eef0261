// Memory-bound token-wise kernels of the attention-server side: RMSNorm (+residual),
// per-head QK RMSNorm + NeoX RoPE + paged KV store, embedding gather, SiLU*mul,
// router scoring + top-k, arg-max sampling, per-token group FP8 quantisation.
// All are written for 16-byte vector access and one pass over HBM.
//
// Reference behaviour: python/minisgl/layers/norm.py (rmsnorm / fused_add_rmsnorm),
// python/minisgl/kernel/csrc/jit/qk_norm_rope.cu:89 (norm + rope + KV store),
// python/minisgl/kernel/csrc/jit/moe_topk_softmax.cu (scoring + top-k + renorm),
// python/minisgl/kernel/csrc/jit/index.cu (embedding gather with shard mask),
// python/minisgl/kernel/csrc/jit/per_token_fp8_packed.cu (1x128 group quant).
#include "common.cuh"

namespace afd {

struct alignas(16) bf16x8 {
  __nv_bfloat162 v[4];
};

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (lane < nw) ? red[lane] : 0.f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

// out = rmsnorm(x [+ residual]) * (w [+ 1]); if residual != null it is updated in place
// to x + residual first (pre-norm residual stream).
template <bool ADD, bool OFFSET1>
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* residual,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                               int H, float eps) {
  extern __shared__ float sbuf[];   // H floats + 32
  float* red = sbuf + H;
  const size_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * H;
  __nv_bfloat16* rr = ADD ? residual + row * H : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    bf16x8 a = *reinterpret_cast<const bf16x8*>(xr + i);
    bf16x8 r;
    if (ADD) r = *reinterpret_cast<const bf16x8*>(rr + i);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 f = __bfloat1622float2(a.v[j]);
      if (ADD) {
        float2 g = __bfloat1622float2(r.v[j]);
        f.x += g.x;
        f.y += g.y;
        // the residual stream is kept in bf16: round once, norm the rounded value
        r.v[j] = __floats2bfloat162_rn(f.x, f.y);
        f = __bfloat1622float2(r.v[j]);
      }
      sbuf[i + 2 * j] = f.x;
      sbuf[i + 2 * j + 1] = f.y;
      ss += f.x * f.x + f.y * f.y;
    }
    if (ADD) *reinterpret_cast<bf16x8*>(rr + i) = r;
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / H + eps);
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    bf16x8 wv = *reinterpret_cast<const bf16x8*>(w + i);
    bf16x8 o;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 g = __bfloat1622float2(wv.v[j]);
      if (OFFSET1) {
        g.x += 1.f;
        g.y += 1.f;
      }
      o.v[j] = __floats2bfloat162_rn(sbuf[i + 2 * j] * inv * g.x, sbuf[i + 2 * j + 1] * inv * g.y);
    }
    *reinterpret_cast<bf16x8*>(out + row * H + i) = o;
  }
}

// One warp per (token, head). Heads [0, Hq) are queries, [Hq, Hq+Hkv) keys,
// [Hq+Hkv, Hq+2Hkv) values. Q and K: optional RMSNorm over head_dim with weight,
// then NeoX RoPE on the first rot_dim dims (pairs (i, i + rot_dim/2)), in place.
// K (after rope) and V are also stored to the paged cache at slot out_loc[token].
template <int D>
__global__ void qk_norm_rope_store_kernel(__nv_bfloat16* qkv, long ld, const __nv_bfloat16* __restrict__ qw,
                                          const __nv_bfloat16* __restrict__ kw,
                                          const float* __restrict__ cos_sin,  // [max_pos][rot_dim]
                                          const int* __restrict__ positions,
                                          const int* __restrict__ out_loc, __nv_bfloat16* k_cache,
                                          __nv_bfloat16* v_cache, int T, int Hq, int Hkv, int rot_dim,
                                          float eps, int max_pos, long cache_slots, int* status) {
  constexpr int PER = D / 32;
  const int heads = Hq + 2 * Hkv;
  const long gw = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  pdl_trigger();
  pdl_wait();
  if (gw >= static_cast<long>(T) * heads) return;
  const int tok = gw / heads, head = gw % heads;
  __nv_bfloat16* p = qkv + static_cast<size_t>(tok) * ld + static_cast<size_t>(head) * D;   // rows `ld` elements apart
  const bool is_q = head < Hq, is_k = !is_q && head < Hq + Hkv;
  // lane holds dims [lane*PER/2 .. ) of the first half and the same of the second half
  // so that rope pairs (i, i + D/2) sit in one lane when rot_dim == D.
  constexpr int HP = PER / 2;
  float lo[HP], hi[HP];
#pragma unroll
  for (int i = 0; i < HP; ++i) {
    lo[i] = __bfloat162float(p[lane * HP + i]);
    hi[i] = __bfloat162float(p[D / 2 + lane * HP + i]);
  }
  if (is_q || is_k) {
    const __nv_bfloat16* w = is_q ? qw : kw;
    if (w != nullptr) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < HP; ++i) ss += lo[i] * lo[i] + hi[i] * hi[i];
      ss = warp_sum(ss);
      const float inv = rsqrtf(ss / D + eps);
#pragma unroll
      for (int i = 0; i < HP; ++i) {
        // round to bf16 after the norm, as a separate norm kernel would
        lo[i] = __bfloat162float(__float2bfloat16(lo[i] * inv * __bfloat162float(w[lane * HP + i])));
        hi[i] = __bfloat162float(__float2bfloat16(hi[i] * inv * __bfloat162float(w[D / 2 + lane * HP + i])));
      }
    }
    int pos = positions[tok];
    if (pos < 0 || pos >= max_pos) {
      set_status(status, kStatusBadExtent);
      pos = 0;
    }
    const float* cs = cos_sin + static_cast<size_t>(pos) * rot_dim;
    const int half = rot_dim / 2;
    if (rot_dim == D) {
#pragma unroll
      for (int i = 0; i < HP; ++i) {
        const int d = lane * HP + i;
        const float c = cs[d], s = cs[half + d];
        const float a = lo[i], b = hi[i];
        lo[i] = a * c - b * s;
        hi[i] = b * c + a * s;
      }
    } else {
      // partial rotary: pairs (d, d + half) for d < half live in the first rot_dim dims.
      // Go through shared-free exchange: write back, then fix up pairs with plain loads.
#pragma unroll
      for (int i = 0; i < HP; ++i) {
        p[lane * HP + i] = __float2bfloat16(lo[i]);
        p[D / 2 + lane * HP + i] = __float2bfloat16(hi[i]);
      }
      __syncwarp();
      for (int d = lane; d < half; d += 32) {
        const float a = __bfloat162float(p[d]), b = __bfloat162float(p[d + half]);
        const float c = cs[d], s = cs[half + d];
        p[d] = __float2bfloat16(a * c - b * s);
        p[d + half] = __float2bfloat16(b * c + a * s);
      }
      __syncwarp();
#pragma unroll
      for (int i = 0; i < HP; ++i) {
        lo[i] = __bfloat162float(p[lane * HP + i]);
        hi[i] = __bfloat162float(p[D / 2 + lane * HP + i]);
      }
    }
#pragma unroll
    for (int i = 0; i < HP; ++i) {
      p[lane * HP + i] = __float2bfloat16(lo[i]);
      p[D / 2 + lane * HP + i] = __float2bfloat16(hi[i]);
    }
  }
  if (!is_q && k_cache != nullptr) {
    const long slot = out_loc[tok];
    if (slot < 0 || slot >= cache_slots) {
      if (slot != -1) set_status(status, kStatusBadExtent);   // -1 = padding token, no store
      return;
    }
    const int kvh = is_k ? head - Hq : head - Hq - Hkv;
    __nv_bfloat16* dst = (is_k ? k_cache : v_cache) + (static_cast<size_t>(slot) * Hkv + kvh) * D;
#pragma unroll
    for (int i = 0; i < HP; ++i) {
      dst[lane * HP + i] = __float2bfloat16(lo[i]);
      dst[D / 2 + lane * HP + i] = __float2bfloat16(hi[i]);
    }
  }
}

__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 __nv_bfloat16* __restrict__ out, int H, int vocab_start, int vocab_end) {
  const int tok = blockIdx.x;
  const int id = ids[tok];
  const bool mine = id >= vocab_start && id < vocab_end;
  const __nv_bfloat16* src = table + static_cast<size_t>(mine ? id - vocab_start : 0) * H;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    uint4 v = mine ? *reinterpret_cast<const uint4*>(src + i) : make_uint4(0, 0, 0, 0);
    *reinterpret_cast<uint4*>(out + static_cast<size_t>(tok) * H + i) = v;
  }
}

__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gate_up, __nv_bfloat16* __restrict__ out,
                                int I) {
  const size_t row = blockIdx.x;
  for (int i = threadIdx.x; i < I; i += blockDim.x) {
    const float g = __bfloat162float(gate_up[row * 2 * I + i]);
    const float u = __bfloat162float(gate_up[row * 2 * I + I + i]);
    out[row * I + i] = __float2bfloat16(silu(g) * u);
  }
}

// Router scoring + top-k, one warp per token, E <= 512.
// scoring 0: softmax over all experts, weights = selected probabilities.
// scoring 1: sigmoid; selection uses score + bias, weights use the un-biased score.
// renorm: divide the selected weights by their sum; scale multiplies the result.
// Ties go to the lower expert index (the order torch.topk gives on equal values is
// not specified; the oracle in the tests uses the same rule).
template <int MAX_PER_LANE, typename LT>
__global__ void topk_route_kernel(const LT* __restrict__ logits, const float* __restrict__ bias,
                                  int* __restrict__ topk_idx, float* __restrict__ topk_w, int T, int E,
                                  int K, int scoring, int renorm, float scale) {
  const int tok = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (tok >= T) return;
  float sc[MAX_PER_LANE], sel[MAX_PER_LANE];
  const LT* lr = logits + static_cast<size_t>(tok) * E;
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < MAX_PER_LANE; ++j) {
    const int e = j * 32 + lane;
    sc[j] = e < E ? static_cast<float>(lr[e]) : -INFINITY;
    mx = fmaxf(mx, sc[j]);
  }
  if (scoring == 0) {
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) {
      const int e = j * 32 + lane;
      sc[j] = e < E ? expf(sc[j] - mx) : 0.f;
      sum += sc[j];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) {
      const int e = j * 32 + lane;
      sc[j] *= inv;
      sel[j] = e < E ? sc[j] : -INFINITY;
    }
  } else {
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) {
      const int e = j * 32 + lane;
      sc[j] = e < E ? 1.f / (1.f + expf(-sc[j])) : 0.f;
      sel[j] = e < E ? sc[j] + (bias ? bias[e] : 0.f) : -INFINITY;
    }
  }
  float wsum = 0.f;
  float my_w = 0.f;
  int my_i = 0;
  for (int k = 0; k < K; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) {
      const int e = j * 32 + lane;
      if (sel[j] > best) {
        best = sel[j];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    float wv = 0.f;
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) {
      if (j * 32 + lane == bi) {
        wv = sc[j];
        sel[j] = -INFINITY;
      }
    }
    wv = warp_sum(wv);   // only the owning lane contributed
    wsum += wv;
    if (lane == k % 32) {
      my_w = wv;
      my_i = bi;
    }
    if (k % 32 == 31 || k == K - 1) {
      // flush up to 32 results (K <= 32 in practice)
      const int base = k - (k % 32);
      if (base + lane <= k) {
        topk_idx[static_cast<size_t>(tok) * K + base + lane] = my_i;
        topk_w[static_cast<size_t>(tok) * K + base + lane] = my_w;
      }
    }
  }
  __syncwarp();
  const float mul = (renorm ? 1.f / fmaxf(wsum, 1e-20f) : 1.f) * scale;
  if (mul != 1.f) {
    for (int k = lane; k < K; k += 32) topk_w[static_cast<size_t>(tok) * K + k] *= mul;
  }
}

// Arg-max over the vocabulary; ties to the lowest index. Two phases so that a handful of
// tokens still fills the GPU: grid (chunks, T) writes one (value, index) candidate per
// chunk, then one CTA per token reduces the candidates.
__device__ __forceinline__ void argmax_combine(float& best, int& bi, float ob, int oi) {
  if (ob > best || (ob == best && oi < bi)) {
    best = ob;
    bi = oi;
  }
}

__device__ __forceinline__ void argmax_block_reduce(float& best, int& bi, float* sv, int* si) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    argmax_combine(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = best;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    best = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      argmax_combine(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
    }
  }
}

template <typename T>
__global__ void argmax_partial_kernel(const T* __restrict__ logits, float* __restrict__ pv, int* __restrict__ pi,
                                      int V, long ld, int chunk) {
  __shared__ float sv[32];
  __shared__ int si[32];
  const T* lr = logits + static_cast<size_t>(blockIdx.y) * ld;
  const int begin = blockIdx.x * chunk, end = min(V, begin + chunk);
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = begin + threadIdx.x; i < end; i += blockDim.x) {
    const float v = static_cast<float>(lr[i]);
    if (v > best) {          // indices grow along the loop: strict > keeps the lowest
      best = v;
      bi = i;
    }
  }
  argmax_block_reduce(best, bi, sv, si);
  if (threadIdx.x == 0) {
    pv[blockIdx.y * gridDim.x + blockIdx.x] = best;
    pi[blockIdx.y * gridDim.x + blockIdx.x] = bi;
  }
}

__global__ void argmax_final_kernel(const float* __restrict__ pv, const int* __restrict__ pi, int* __restrict__ out,
                                    int chunks) {
  __shared__ float sv[32];
  __shared__ int si[32];
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < chunks; i += blockDim.x) {
    argmax_combine(best, bi, pv[blockIdx.x * chunks + i], pi[blockIdx.x * chunks + i]);
  }
  argmax_block_reduce(best, bi, sv, si);
  if (threadIdx.x == 0) out[blockIdx.x] = bi;
}

// Per-token, per-`group`-wide FP8 e4m3 quantisation. scale = amax/448 floored at
// 1e-10/448; pow2 != 0 rounds the scale up to a power of two (UE8M0-compatible).
// One warp per (row, group of 128) or per (row, 4 groups of 32).
__global__ void group_quant_fp8_kernel(const __nv_bfloat16* __restrict__ x, uint8_t* __restrict__ q,
                                       float* __restrict__ s, long rows, int H, int group, int pow2) {
  const long gw = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int chunks = H / 128;
  if (gw >= rows * chunks) return;
  const long row = gw / chunks;
  const int ch = gw % chunks;
  const __nv_bfloat16* src = x + row * H + ch * 128 + lane * 4;
  float v[4];
  const uint2 raw = *reinterpret_cast<const uint2*>(src);
  const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
  float2 f0 = __bfloat1622float2(b2[0]), f1 = __bfloat1622float2(b2[1]);
  v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
  float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
  const int span = group / 4;   // lanes per group: 32 (group 128) or 8 (group 32)
  for (int o = span / 2; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float scale = fmaxf(amax, 1e-10f) / 448.f;
  if (pow2) scale = exp2f(ceilf(log2f(scale)));
  const float inv = 1.f / scale;
  uint32_t packed = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(v[i] * inv, __NV_SATFINITE, __NV_E4M3)) << (8 * i);
  }
  *reinterpret_cast<uint32_t*>(q + row * H + ch * 128 + lane * 4) = packed;
  if ((lane % span) == 0) s[row * (H / group) + ch * (128 / group) + lane / span] = scale;
}

}  // namespace afd

using namespace afd;

extern "C" int afd_rmsnorm(const void* x, void* residual, const void* w, void* out, long rows, int H,
                           float eps, int offset1, void* stream) {
  if (H % 8 != 0) return -1;
  if (rows == 0) return 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int threads = H / 8 >= 512 ? 512 : (H / 8 >= 256 ? 256 : 128);
  const size_t smem = (H + 32) * sizeof(float);
  auto x_ = static_cast<const __nv_bfloat16*>(x);
  auto r_ = static_cast<__nv_bfloat16*>(residual);
  auto w_ = static_cast<const __nv_bfloat16*>(w);
  auto o_ = static_cast<__nv_bfloat16*>(out);
  if (residual) {
    if (offset1) rmsnorm_kernel<true, true><<<rows, threads, smem, st>>>(x_, r_, w_, o_, H, eps);
    else rmsnorm_kernel<true, false><<<rows, threads, smem, st>>>(x_, r_, w_, o_, H, eps);
  } else {
    if (offset1) rmsnorm_kernel<false, true><<<rows, threads, smem, st>>>(x_, r_, w_, o_, H, eps);
    else rmsnorm_kernel<false, false><<<rows, threads, smem, st>>>(x_, r_, w_, o_, H, eps);
  }
  AFD_CHECK_LAUNCH();
  return 0;
}

extern "C" int afd_qk_norm_rope_store(void* qkv, long ld, const void* qw, const void* kw, const void* cos_sin,
                                      const void* positions, const void* out_loc, void* k_cache,
                                      void* v_cache, int T, int Hq, int Hkv, int D, int rot_dim,
                                      float eps, int max_pos, long cache_slots, void* status,
                                      void* stream) {
  if (T == 0) return 0;
  if (rot_dim > D || rot_dim % 2 != 0 || ld < static_cast<long>(Hq + 2 * Hkv) * D) return -1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long warps = static_cast<long>(T) * (Hq + 2 * Hkv);
  const int threads = 256;
  const int blocks = static_cast<int>((warps * 32 + threads - 1) / threads);
  cudaError_t le = cudaSuccess;
#define LAUNCH_QK(DD)                                                                                   \
  le = launch_pdl(qk_norm_rope_store_kernel<DD>, dim3(blocks), dim3(threads), 0, st, 1,                 \
      static_cast<__nv_bfloat16*>(qkv), ld, static_cast<const __nv_bfloat16*>(qw),                      \
      static_cast<const __nv_bfloat16*>(kw), static_cast<const float*>(cos_sin),                        \
      static_cast<const int*>(positions), static_cast<const int*>(out_loc),                             \
      static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), T, Hq, Hkv, rot_dim,  \
      eps, max_pos, cache_slots, static_cast<int*>(status))
  if (D == 128) LAUNCH_QK(128);
  else if (D == 256) LAUNCH_QK(256);
  else if (D == 64) LAUNCH_QK(64);
  else return -2;
#undef LAUNCH_QK
  if (le != cudaSuccess) return static_cast<int>(le);
  return 0;
}

extern "C" int afd_embedding(const void* ids, const void* table, void* out, int T, int H, int vocab_start,
                             int vocab_end, void* stream) {
  if (T == 0) return 0;
  if (H % 8 != 0) return -1;
  embedding_kernel<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const int*>(ids), static_cast<const __nv_bfloat16*>(table),
      static_cast<__nv_bfloat16*>(out), H, vocab_start, vocab_end);
  AFD_CHECK_LAUNCH();
  return 0;
}

extern "C" int afd_silu_mul(const void* gate_up, void* out, long rows, int I, void* stream) {
  if (rows == 0) return 0;
  silu_mul_kernel<<<rows, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(gate_up), static_cast<__nv_bfloat16*>(out), I);
  AFD_CHECK_LAUNCH();
  return 0;
}

template <typename LT>
static void launch_topk(const void* logits, const float* b, int* ti, float* tw, int T, int E, int K, int scoring,
                        int renorm, float scale, cudaStream_t st) {
  const int threads = 128;
  const int blocks = (T * 32 + threads - 1) / threads;
  auto l = static_cast<const LT*>(logits);
  if (E <= 128) topk_route_kernel<4, LT><<<blocks, threads, 0, st>>>(l, b, ti, tw, T, E, K, scoring, renorm, scale);
  else if (E <= 256) topk_route_kernel<8, LT><<<blocks, threads, 0, st>>>(l, b, ti, tw, T, E, K, scoring, renorm, scale);
  else topk_route_kernel<16, LT><<<blocks, threads, 0, st>>>(l, b, ti, tw, T, E, K, scoring, renorm, scale);
}

extern "C" int afd_topk_route(const void* logits, const void* bias, void* topk_idx, void* topk_w, int T,
                              int E, int K, int scoring, int renorm, float scale, int logits_bf16,
                              void* stream) {
  if (T == 0) return 0;
  if (E > 512 || K > 32 || K > E) return -1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto b = static_cast<const float*>(bias);
  auto ti = static_cast<int*>(topk_idx);
  auto tw = static_cast<float*>(topk_w);
  if (logits_bf16) launch_topk<__nv_bfloat16>(logits, b, ti, tw, T, E, K, scoring, renorm, scale, st);
  else launch_topk<float>(logits, b, ti, tw, T, E, K, scoring, renorm, scale, st);
  AFD_CHECK_LAUNCH();
  return 0;
}

// scratch: at least T * afd_argmax_chunks(V) * 8 bytes (candidate values, then indices).
extern "C" int afd_argmax_chunks(int V) {
  const int c = (V + 4095) / 4096;
  return c < 1 ? 1 : c;
}

extern "C" int afd_argmax(const void* logits, void* out, int T, int V, long ld, int is_bf16, void* scratch,
                          void* stream) {
  if (T == 0) return 0;
  if (scratch == nullptr) return -1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int chunks = afd_argmax_chunks(V);
  const int chunk = (V + chunks - 1) / chunks;
  float* pv = static_cast<float*>(scratch);
  int* pi = reinterpret_cast<int*>(pv + static_cast<size_t>(T) * chunks);
  dim3 grid(chunks, T);
  if (is_bf16) argmax_partial_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(logits), pv, pi, V, ld, chunk);
  else argmax_partial_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(logits), pv, pi, V, ld, chunk);
  AFD_CHECK_LAUNCH();
  argmax_final_kernel<<<T, 64, 0, st>>>(pv, pi, static_cast<int*>(out), chunks);
  AFD_CHECK_LAUNCH();
  return 0;
}

extern "C" int afd_group_quant_fp8(const void* x, void* q, void* s, long rows, int H, int group, int pow2,
                                   void* stream) {
  if (rows == 0) return 0;
  if (H % 128 != 0 || (group != 128 && group != 32)) return -1;
  const long warps = rows * (H / 128);
  const int threads = 256;
  const int blocks = static_cast<int>((warps * 32 + threads - 1) / threads);
  group_quant_fp8_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<uint8_t*>(q), static_cast<float*>(s), rows, H,
      group, pow2);
  AFD_CHECK_LAUNCH();
  return 0;
}
