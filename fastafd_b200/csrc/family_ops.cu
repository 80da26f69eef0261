// Kernels that only some model families need, so that those families stay on the same fused
// decode path as Qwen3-MoE instead of falling back to framework ops:
//
//   cross_head_norm_rope_store_kernel  MiniMax-M2: RMSNorm over ALL q heads jointly (and all k heads
//       jointly), then RoPE (partial rotary) and the paged K/V store, one CTA per token. Under tensor
//       parallelism the sums of squares come in from an all-reduce (qk_square_sums_kernel makes the
//       local ones). Reference: python/minisgl/kernel/csrc/jit/minimax_qk_norm.cu:78,119,257.
//   grouped_topk_route_kernel  GLM-4 / DeepSeek routing: sigmoid scores + selection bias, groups
//       ranked by the sum of their two best biased scores, top-k inside the chosen groups.
//       Reference: python/minisgl/models/glm4_moe.py:108-153.
//   shared_gate_mul_kernel  Qwen3.5: shared-expert output scaled by sigmoid(x . w_gate), the GEMV
//       and the scaling in one launch. Reference: python/minisgl/kernel/qwen35_shared_gate.py:33-84.
//   sigmoid_gate_mul_kernel  Qwen3.5 gated attention: o *= sigmoid(gate), gate read in place from
//       the merged projection output (row stride), no fp32 temporaries.
#include "common.cuh"

namespace afd {

// ------------------------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(256) cross_head_norm_rope_store_kernel(
    __nv_bfloat16* qkv, long ld, const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
    const float* __restrict__ sq_in, float q_denom, float k_denom, const float* __restrict__ cos_sin,
    const int* __restrict__ positions, const int* __restrict__ out_loc, __nv_bfloat16* k_cache,
    __nv_bfloat16* v_cache, int Hq, int Hkv, int rot_dim, float eps, int max_pos, long cache_slots, int* status) {
  constexpr int PER = D / 32, HP = PER / 2;
  const int tok = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __nv_bfloat16* row = qkv + static_cast<size_t>(tok) * ld;
  __shared__ float s_red[2][8];
  __shared__ float s_inv[2];
  if (sq_in == nullptr) {
    float sq = 0.f, sk = 0.f;
    for (int h = warp; h < Hq + Hkv; h += nw) {
      const __nv_bfloat16* p = row + h * D;
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const float v = __bfloat162float(p[lane * PER + i]);
        ss += v * v;
      }
      if (h < Hq) sq += ss; else sk += ss;
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    if (lane == 0) {
      s_red[0][warp] = sq;
      s_red[1][warp] = sk;
    }
    __syncthreads();
    if (threadIdx.x < 2) {
      float t = 0.f;
      for (int w = 0; w < nw; ++w) t += s_red[threadIdx.x][w];
      s_inv[threadIdx.x] = rsqrtf(t / (threadIdx.x == 0 ? q_denom : k_denom) + eps);
    }
  } else if (threadIdx.x < 2) {
    s_inv[threadIdx.x] = rsqrtf(sq_in[tok * 2 + threadIdx.x] / (threadIdx.x == 0 ? q_denom : k_denom) + eps);
  }
  __syncthreads();
  int pos = positions[tok];
  if (pos < 0 || pos >= max_pos) {
    if (threadIdx.x == 0) set_status(status, kStatusBadExtent);
    pos = 0;
  }
  const float* cs = cos_sin + static_cast<size_t>(pos) * rot_dim;
  const int half = rot_dim / 2;
  const long slot = k_cache != nullptr ? out_loc[tok] : -1;
  for (int h = warp; h < Hq + 2 * Hkv; h += nw) {
    __nv_bfloat16* p = row + h * D;
    const bool is_q = h < Hq, is_k = !is_q && h < Hq + Hkv;
    float lo[HP], hi[HP];
#pragma unroll
    for (int i = 0; i < HP; ++i) {
      lo[i] = __bfloat162float(p[lane * HP + i]);
      hi[i] = __bfloat162float(p[D / 2 + lane * HP + i]);
    }
    if (is_q || is_k) {
      const float inv = s_inv[is_q ? 0 : 1];
      const __nv_bfloat16* w = is_q ? qw + h * D : kw + (h - Hq) * D;
#pragma unroll
      for (int i = 0; i < HP; ++i) {
        lo[i] = __bfloat162float(__float2bfloat16(lo[i] * inv * __bfloat162float(w[lane * HP + i])));
        hi[i] = __bfloat162float(__float2bfloat16(hi[i] * inv * __bfloat162float(w[D / 2 + lane * HP + i])));
      }
      if (rot_dim == D) {
#pragma unroll
        for (int i = 0; i < HP; ++i) {
          const int d = lane * HP + i;
          const float c = cs[d], s = cs[half + d];
          const float a = lo[i], b = hi[i];
          lo[i] = a * c - b * s;
          hi[i] = b * c + a * s;
        }
#pragma unroll
        for (int i = 0; i < HP; ++i) {
          p[lane * HP + i] = __float2bfloat16(lo[i]);
          p[D / 2 + lane * HP + i] = __float2bfloat16(hi[i]);
        }
      } else {
        // partial rotary: pairs (d, d + half), d < half, all inside the first rot_dim dims
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
    }
    if (!is_q && k_cache != nullptr) {
      if (slot < 0 || slot >= cache_slots) {
        if (slot != -1 && lane == 0) set_status(status, kStatusBadExtent);     // -1 = padding token
        continue;
      }
      const int kvh = is_k ? h - Hq : h - Hq - Hkv;
      __nv_bfloat16* dst = (is_k ? k_cache : v_cache) + (static_cast<size_t>(slot) * Hkv + kvh) * D;
#pragma unroll
      for (int i = 0; i < HP; ++i) {
        dst[lane * HP + i] = __float2bfloat16(lo[i]);
        dst[D / 2 + lane * HP + i] = __float2bfloat16(hi[i]);
      }
    }
  }
}

// [T][2] fp32: sum of squares over this rank's q heads and k heads (input of the TP all-reduce).
__global__ void __launch_bounds__(256) qk_square_sums_kernel(const __nv_bfloat16* __restrict__ qkv, long ld,
                                                            float* __restrict__ out, int q_elems, int k_elems) {
  const int tok = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const __nv_bfloat16* row = qkv + static_cast<size_t>(tok) * ld;
  __shared__ float s_red[2][8];
  float sq = 0.f, sk = 0.f;
  for (int i = threadIdx.x; i < q_elems + k_elems; i += blockDim.x) {
    const float v = __bfloat162float(row[i]);
    if (i < q_elems) sq += v * v; else sk += v * v;
  }
  sq = warp_sum(sq);
  sk = warp_sum(sk);
  if (lane == 0) {
    s_red[0][warp] = sq;
    s_red[1][warp] = sk;
  }
  __syncthreads();
  if (threadIdx.x < 2) {
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += s_red[threadIdx.x][w];
    out[tok * 2 + threadIdx.x] = t;
  }
}

// ------------------------------------------------------------------------------------------
// One warp per token; E <= 512, n_group <= 32, E % n_group == 0, group size >= 2.
constexpr int kGroupedMaxE = 512;

template <typename LT>
__global__ void __launch_bounds__(128) grouped_topk_route_kernel(const LT* __restrict__ logits, const float* __restrict__ bias,
                                                                int* __restrict__ topk_idx, float* __restrict__ topk_w,
                                                                int T, int E, int K, int n_group, int topk_group,
                                                                int renorm, float scale) {
  __shared__ float s_sc[4][kGroupedMaxE];
  __shared__ float s_sel[4][kGroupedMaxE];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + warp;
  if (t >= T) return;
  float* sc = s_sc[warp];
  float* sel = s_sel[warp];
  for (int e = lane; e < E; e += 32) {
    const float v = 1.f / (1.f + expf(-static_cast<float>(logits[static_cast<size_t>(t) * E + e])));
    sc[e] = v;
    sel[e] = v + (bias ? bias[e] : 0.f);
  }
  __syncwarp();
  // group score = sum of the group's two best biased scores
  const int gs = E / n_group;
  float gscore = -INFINITY;
  if (lane < n_group) {
    float b1 = -INFINITY, b2 = -INFINITY;
    for (int i = 0; i < gs; ++i) {
      const float v = sel[lane * gs + i];
      if (v > b1) {
        b2 = b1;
        b1 = v;
      } else if (v > b2) {
        b2 = v;
      }
    }
    gscore = b1 + b2;
  }
  // choose topk_group groups (ties: lowest group index)
  uint32_t gmask = 0;
  for (int r = 0; r < topk_group; ++r) {
    float best = gscore;
    int bi = lane < n_group ? lane : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (bi < 32) gmask |= 1u << bi;
    if (lane == bi) gscore = -INFINITY;
  }
  for (int e = lane; e < E; e += 32) {
    if (!((gmask >> (e / gs)) & 1u)) sel[e] = -INFINITY;
  }
  __syncwarp();
  // top-K among the remaining experts (value descending, index ascending)
  float wsum = 0.f, my_w = 0.f;
  int my_i = 0;
  for (int k = 0; k < K; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int e = lane; e < E; e += 32) {
      const float v = sel[e];
      if (v > best) {
        best = v;
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
    if (bi >= E) bi = 0;                      // fewer candidates than K (cannot happen for valid configs)
    const float wv = sc[bi];
    wsum += wv;
    if (lane == k) {
      my_w = wv;
      my_i = bi;
    }
    __syncwarp();
    if (lane == 0) sel[bi] = -INFINITY;
    __syncwarp();
  }
  const float mul = (renorm ? 1.f / fmaxf(wsum, 1e-20f) : 1.f) * scale;
  if (lane < K) {
    topk_idx[static_cast<size_t>(t) * K + lane] = my_i;
    topk_w[static_cast<size_t>(t) * K + lane] = my_w * mul;
  }
}

// ------------------------------------------------------------------------------------------
// y[t, :] *= sigmoid(dot(x[t, :], gw)), one CTA per token.
__global__ void __launch_bounds__(256) shared_gate_mul_kernel(const __nv_bfloat16* __restrict__ x,
                                                             const __nv_bfloat16* __restrict__ gw,
                                                             __nv_bfloat16* y, int H) {
  const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __shared__ float s_red[8];
  __shared__ float s_g;
  const __nv_bfloat16* xr = x + static_cast<size_t>(t) * H;
  float acc = 0.f;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    const uint4 xa = *reinterpret_cast<const uint4*>(xr + i);
    const uint4 ga = *reinterpret_cast<const uint4*>(gw + i);
    const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xa);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&ga);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 xv = __bfloat1622float2(x2[j]), gv = __bfloat1622float2(g2[j]);
      acc = fmaf(xv.x, gv.x, acc);
      acc = fmaf(xv.y, gv.y, acc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) s_red[warp] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tsum = 0.f;
    for (int w = 0; w < nw; ++w) tsum += s_red[w];
    // the gate projection's output is a bf16 tensor in the unfused form: round before the sigmoid
    tsum = __bfloat162float(__float2bfloat16(tsum));
    s_g = 1.f / (1.f + expf(-tsum));
  }
  __syncthreads();
  const float g = s_g;
  __nv_bfloat16* yr = y + static_cast<size_t>(t) * H;
  for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
    uint4 ya = *reinterpret_cast<const uint4*>(yr + i);
    __nv_bfloat162* y2 = reinterpret_cast<__nv_bfloat162*>(&ya);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 v = __bfloat1622float2(y2[j]);
      y2[j] = __floats2bfloat162_rn(v.x * g, v.y * g);
    }
    *reinterpret_cast<uint4*>(yr + i) = ya;
  }
}

// o[t, i] *= sigmoid(gate[t, i]); o contiguous [T][n], gate rows `gate_ld` elements apart.
__global__ void sigmoid_gate_mul_kernel(__nv_bfloat16* o, const __nv_bfloat16* __restrict__ gate, long gate_ld,
                                        long T, int n) {
  const long vec_per_row = n / 8;
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= T * vec_per_row) return;
  const long t = idx / vec_per_row, c = idx - t * vec_per_row;
  uint4 oa = *reinterpret_cast<const uint4*>(o + t * n + c * 8);
  const uint4 ga = *reinterpret_cast<const uint4*>(gate + t * gate_ld + c * 8);
  __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&oa);
  const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&ga);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 ov = __bfloat1622float2(o2[j]), gv = __bfloat1622float2(g2[j]);
    o2[j] = __floats2bfloat162_rn(ov.x / (1.f + expf(-gv.x)), ov.y / (1.f + expf(-gv.y)));
  }
  *reinterpret_cast<uint4*>(o + t * n + c * 8) = oa;
}

}  // namespace afd

using namespace afd;

extern "C" int afd_cross_head_norm_rope_store(void* qkv, long ld, const void* qw, const void* kw, const void* sq_in,
                                              float q_denom, float k_denom, const void* cos_sin, const void* positions,
                                              const void* out_loc, void* k_cache, void* v_cache, int T, int Hq, int Hkv,
                                              int D, int rot_dim, float eps, int max_pos, long cache_slots,
                                              void* status, void* stream) {
  if (T == 0) return 0;
  if (rot_dim % 2 != 0 || rot_dim > D || ld < static_cast<long>(Hq + 2 * Hkv) * D) return -1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define LAUNCH_XH(DD)                                                                                          \
  cross_head_norm_rope_store_kernel<DD><<<T, 256, 0, st>>>(                                                     \
      static_cast<__nv_bfloat16*>(qkv), ld, static_cast<const __nv_bfloat16*>(qw),                              \
      static_cast<const __nv_bfloat16*>(kw), static_cast<const float*>(sq_in), q_denom, k_denom,                \
      static_cast<const float*>(cos_sin), static_cast<const int*>(positions), static_cast<const int*>(out_loc), \
      static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), Hq, Hkv, rot_dim, eps,        \
      max_pos, cache_slots, static_cast<int*>(status))
  if (D == 128) LAUNCH_XH(128);
  else if (D == 256) LAUNCH_XH(256);
  else if (D == 64) LAUNCH_XH(64);
  else return -2;
#undef LAUNCH_XH
  AFD_CHECK_LAUNCH();
  return 0;
}

extern "C" int afd_qk_square_sums(const void* qkv, long ld, void* out, int T, int q_elems, int k_elems, void* stream) {
  if (T == 0) return 0;
  qk_square_sums_kernel<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(qkv), ld, static_cast<float*>(out), q_elems, k_elems);
  AFD_CHECK_LAUNCH();
  return 0;
}

extern "C" int afd_grouped_topk_route(const void* logits, const void* bias, void* topk_idx, void* topk_w, int T, int E,
                                      int K, int n_group, int topk_group, int renorm, float scale, int logits_bf16,
                                      void* stream) {
  if (T == 0) return 0;
  if (E > kGroupedMaxE || n_group < 1 || n_group > 32 || E % n_group != 0 || E / n_group < 2 || K > 32 ||
      topk_group < 1 || topk_group > n_group || K > topk_group * (E / n_group))
    return -1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int grid = (T + 3) / 4;
  if (logits_bf16) {
    grouped_topk_route_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(
        static_cast<const __nv_bfloat16*>(logits), static_cast<const float*>(bias), static_cast<int*>(topk_idx),
        static_cast<float*>(topk_w), T, E, K, n_group, topk_group, renorm, scale);
  } else {
    grouped_topk_route_kernel<float><<<grid, 128, 0, st>>>(
        static_cast<const float*>(logits), static_cast<const float*>(bias), static_cast<int*>(topk_idx),
        static_cast<float*>(topk_w), T, E, K, n_group, topk_group, renorm, scale);
  }
  AFD_CHECK_LAUNCH();
  return 0;
}

extern "C" int afd_shared_gate_mul(const void* x, const void* gw, void* y, int T, int H, void* stream) {
  if (T == 0) return 0;
  if (H % 8 != 0) return -1;
  shared_gate_mul_kernel<<<T, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(gw), static_cast<__nv_bfloat16*>(y), H);
  AFD_CHECK_LAUNCH();
  return 0;
}

extern "C" int afd_sigmoid_gate_mul(void* o, const void* gate, long gate_ld, long T, int n, void* stream) {
  if (T == 0) return 0;
  if (n % 8 != 0 || gate_ld % 8 != 0) return -1;
  const long total = T * (n / 8);
  sigmoid_gate_mul_kernel<<<static_cast<unsigned int>((total + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__nv_bfloat16*>(o), static_cast<const __nv_bfloat16*>(gate), gate_ld, T, n);
  AFD_CHECK_LAUNCH();
  return 0;
}
