// Gated DeltaNet decode step (Qwen3.5 hybrid linear-attention layers), one token per request:
//
//   1. depthwise causal conv over the last W inputs of every channel (+ SiLU), shifting the
//      per-request tap state in place;
//   2. gated delta rule on the fp32 recurrent state S[Hv][Dv][Dk] of the request:
//        g = -exp(A_log) * softplus(a + dt_bias);  beta = sigmoid(b)
//        S *= exp(g);  delta = (v - S k) * beta;  S += delta (x) k;  o = S q * Dk^-0.5
//      with q, k L2-normalised per head (q/k heads are shared by Hv/Hk value heads);
//   3. per-head gated RMSNorm: out = rmsnorm(o) * w * silu(z).
//
// The op is bound by streaming the state (Dv*Dk*4 bytes per value head, read and written
// once): one CTA per (token, value head), one warp per state row, 16-byte accesses.
//
// Reference behaviour: python/minisgl/kernel/qwen35_gdn.py:235-318 (conv step), :565-652
// (recurrent update), python/minisgl/kernel/qwen35_gated_norm.py:28 (gated norm).
#include "common.cuh"

namespace afd {

__global__ void gdn_conv_step_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                     const __nv_bfloat16* __restrict__ w,   // [C][W]
                                     __nv_bfloat16* conv_state,             // [slots][W-1][C]
                                     const int* __restrict__ slots, int T, int C, int W, int num_slots,
                                     int* status, long x_ld) {
  const int t = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int slot = slots[t];
  if (slot < 0 || slot >= num_slots) {
    set_status(status, kStatusBadExtent);
    return;
  }
  __nv_bfloat16* st = conv_state + static_cast<size_t>(slot) * (W - 1) * C + c;
  const float xin = __bfloat162float(x[static_cast<size_t>(t) * x_ld + c]);
  float acc = xin * __bfloat162float(w[c * W + W - 1]);
  float prev[8];
  for (int i = 0; i < W - 1; ++i) {
    prev[i] = __bfloat162float(st[static_cast<size_t>(i) * C]);
    acc += prev[i] * __bfloat162float(w[c * W + i]);
  }
  for (int i = 0; i + 1 < W - 1; ++i) st[static_cast<size_t>(i) * C] = __float2bfloat16(prev[i + 1]);
  st[static_cast<size_t>(W - 2) * C] = __float2bfloat16(xin);
  y[static_cast<size_t>(t) * C + c] = __float2bfloat16(silu(acc));
}

template <int DK>
__global__ void __launch_bounds__(256) gdn_recurrent_kernel(
    const __nv_bfloat16* __restrict__ qkv,   // [T][2*Hk*DK + Hv*Dv] after conv
    const __nv_bfloat16* __restrict__ z,     // [T][Hv*Dv]
    const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b,   // [T][Hv]
    const float* __restrict__ A_log, const float* __restrict__ dt_bias,         // [Hv]
    const __nv_bfloat16* __restrict__ norm_w,                                   // [Dv]
    float* rec_state,                        // [slots][Hv][Dv][DK]
    const int* __restrict__ slots, __nv_bfloat16* __restrict__ out, int T, int Hk, int Hv, int Dv, int num_slots,
    float eps, int* status, long z_ld, long a_ld, long b_ld) {
  constexpr int PER = DK / 32;
  const int t = blockIdx.y, h = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __shared__ float s_o[256];
  __shared__ float s_red[8];
  const int slot = slots[t];
  if (slot < 0 || slot >= num_slots) {
    if (threadIdx.x == 0) set_status(status, kStatusBadExtent);
    return;
  }
  const int C = 2 * Hk * DK + Hv * Dv;
  const int hk = h / (Hv / Hk);
  const __nv_bfloat16* row = qkv + static_cast<size_t>(t) * C;
  float q[PER], k[PER];
  float qs = 0.f, ks = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    q[i] = __bfloat162float(row[hk * DK + lane * PER + i]);
    k[i] = __bfloat162float(row[Hk * DK + hk * DK + lane * PER + i]);
    qs += q[i] * q[i];
    ks += k[i] * k[i];
  }
  qs = warp_sum(qs);
  ks = warp_sum(ks);
  const float qn = rsqrtf(qs + 1e-6f) * rsqrtf(static_cast<float>(DK));
  const float kn = rsqrtf(ks + 1e-6f);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    q[i] *= qn;
    k[i] *= kn;
  }
  const float av = __bfloat162float(a[static_cast<size_t>(t) * a_ld + h]) + dt_bias[h];
  const float sp = av > 20.f ? av : log1pf(expf(av));
  const float decay = expf(-expf(A_log[h]) * sp);
  const float beta = 1.f / (1.f + expf(-__bfloat162float(b[static_cast<size_t>(t) * b_ld + h])));
  float* S = rec_state + (static_cast<size_t>(slot) * Hv + h) * Dv * DK;
  const __nv_bfloat16* vrow = row + 2 * Hk * DK + h * Dv;
  for (int r = warp; r < Dv; r += nw) {
    float* sr = S + static_cast<size_t>(r) * DK + lane * PER;
    float s[PER];
    float kv = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      s[i] = sr[i] * decay;
      kv += s[i] * k[i];
    }
    kv = warp_sum(kv);
    const float delta = (__bfloat162float(vrow[r]) - kv) * beta;
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      s[i] += delta * k[i];
      o += s[i] * q[i];
      sr[i] = s[i];
    }
    o = warp_sum(o);
    if (lane == 0) s_o[r] = __bfloat162float(__float2bfloat16(o));   // the op's output dtype is bf16
  }
  __syncthreads();
  // gated RMSNorm over the head's Dv outputs
  float ss = 0.f;
  for (int r = threadIdx.x; r < Dv; r += blockDim.x) ss += s_o[r] * s_o[r];
  ss = warp_sum(ss);
  if (lane == 0) s_red[warp] = ss;
  __syncthreads();
  float tot = lane < nw ? s_red[lane] : 0.f;
  tot = warp_sum(tot);
  const float inv = rsqrtf(tot / Dv + eps);
  for (int r = threadIdx.x; r < Dv; r += blockDim.x) {
    const float zz = __bfloat162float(z[static_cast<size_t>(t) * z_ld + static_cast<size_t>(h) * Dv + r]);
    out[(static_cast<size_t>(t) * Hv + h) * Dv + r] =
        __float2bfloat16(s_o[r] * inv * __bfloat162float(norm_w[r]) * silu(zz));
  }
}

// ---------------------------------------------------------------------------------------
// Prefill (token-serial, like the reference's path on this architecture:
// python/minisgl/kernel/qwen35_gdn.py:443-513). Sequences are given by cu_seqlens; a sequence
// flagged fresh starts from zero state, otherwise from its slot's state. The recurrent state
// rows stay in registers across the whole sequence and are written back once.
// ---------------------------------------------------------------------------------------
__global__ void gdn_conv_prefill_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                        const __nv_bfloat16* __restrict__ w, __nv_bfloat16* conv_state,
                                        const int* __restrict__ slots, const int* __restrict__ cu_seqlens,
                                        const int* __restrict__ fresh, int C, int W, int num_slots, int* status) {
  const int s = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int slot = slots[s];
  if (slot < 0 || slot >= num_slots) {
    set_status(status, kStatusBadExtent);
    return;
  }
  const int t0 = cu_seqlens[s], t1 = cu_seqlens[s + 1];
  if (t1 <= t0) return;
  __nv_bfloat16* st = conv_state + static_cast<size_t>(slot) * (W - 1) * C + c;
  float win[8], wt[9];
  for (int i = 0; i < W - 1; ++i) win[i] = fresh[s] ? 0.f : __bfloat162float(st[static_cast<size_t>(i) * C]);
  for (int i = 0; i < W; ++i) wt[i] = __bfloat162float(w[c * W + i]);
  for (int t = t0; t < t1; ++t) {
    const float xin = __bfloat162float(x[static_cast<size_t>(t) * C + c]);
    float acc = xin * wt[W - 1];
    for (int i = 0; i < W - 1; ++i) acc += win[i] * wt[i];
    for (int i = 0; i + 1 < W - 1; ++i) win[i] = win[i + 1];
    win[W - 2] = xin;
    y[static_cast<size_t>(t) * C + c] = __float2bfloat16(silu(acc));
  }
  for (int i = 0; i < W - 1; ++i) st[static_cast<size_t>(i) * C] = __float2bfloat16(win[i]);
}

// One CTA per (value head, sequence), 8 warps; warp w owns state rows w, w+8, ... (RPW rows).
template <int DK, int RPW>
__global__ void __launch_bounds__(256) gdn_recurrent_prefill_kernel(
    const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b,
    const float* __restrict__ A_log, const float* __restrict__ dt_bias, float* rec_state,
    const int* __restrict__ slots, const int* __restrict__ cu_seqlens, const int* __restrict__ fresh,
    __nv_bfloat16* __restrict__ o_raw,       // [T][Hv][Dv] un-normalised outputs (bf16, as in decode)
    int Hk, int Hv, int Dv, int num_slots, int* status) {
  constexpr int PER = DK / 32;
  const int h = blockIdx.x, s = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slot = slots[s];
  if (slot < 0 || slot >= num_slots) {
    if (threadIdx.x == 0) set_status(status, kStatusBadExtent);
    return;
  }
  const int t0 = cu_seqlens[s], t1 = cu_seqlens[s + 1];
  if (t1 <= t0) return;
  const int C = 2 * Hk * DK + Hv * Dv;
  const int hk = h / (Hv / Hk);
  float* S = rec_state + (static_cast<size_t>(slot) * Hv + h) * Dv * DK;
  float st[RPW][PER];
#pragma unroll
  for (int j = 0; j < RPW; ++j) {
    const int r = warp + j * 8;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      st[j][i] = (r < Dv && !fresh[s]) ? S[static_cast<size_t>(r) * DK + lane * PER + i] : 0.f;
  }
  const float neg_a = -expf(A_log[h]), bias = dt_bias[h];
  for (int t = t0; t < t1; ++t) {
    const __nv_bfloat16* row = qkv + static_cast<size_t>(t) * C;
    float q[PER], k[PER];
    float qs = 0.f, ks = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      q[i] = __bfloat162float(row[hk * DK + lane * PER + i]);
      k[i] = __bfloat162float(row[Hk * DK + hk * DK + lane * PER + i]);
      qs += q[i] * q[i];
      ks += k[i] * k[i];
    }
    qs = warp_sum(qs);
    ks = warp_sum(ks);
    const float qn = rsqrtf(qs + 1e-6f) * rsqrtf(static_cast<float>(DK));
    const float kn = rsqrtf(ks + 1e-6f);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      q[i] *= qn;
      k[i] *= kn;
    }
    const float av = __bfloat162float(a[static_cast<size_t>(t) * Hv + h]) + bias;
    const float sp = av > 20.f ? av : log1pf(expf(av));
    const float decay = expf(neg_a * sp);
    const float beta = 1.f / (1.f + expf(-__bfloat162float(b[static_cast<size_t>(t) * Hv + h])));
    const __nv_bfloat16* vrow = row + 2 * Hk * DK + h * Dv;
    float kv[RPW];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      kv[j] = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        st[j][i] *= decay;
        kv[j] += st[j][i] * k[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int j = 0; j < RPW; ++j) kv[j] += __shfl_xor_sync(0xffffffffu, kv[j], o);
    }
    float ov[RPW];
#pragma unroll
    for (int j = 0; j < RPW; ++j) {
      const int r = warp + j * 8;
      const float delta = ((r < Dv ? __bfloat162float(vrow[r]) : 0.f) - kv[j]) * beta;
      ov[j] = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        st[j][i] += delta * k[i];
        ov[j] += st[j][i] * q[i];
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
      for (int j = 0; j < RPW; ++j) ov[j] += __shfl_xor_sync(0xffffffffu, ov[j], o);
    }
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < RPW; ++j) {
        const int r = warp + j * 8;
        if (r < Dv) o_raw[(static_cast<size_t>(t) * Hv + h) * Dv + r] = __float2bfloat16(ov[j]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < RPW; ++j) {
    const int r = warp + j * 8;
    if (r < Dv) {
#pragma unroll
      for (int i = 0; i < PER; ++i) S[static_cast<size_t>(r) * DK + lane * PER + i] = st[j][i];
    }
  }
}

// out[t][h][:] = rmsnorm(o_raw[t][h][:]) * w * silu(z[t][h][:]); rows at or past n_valid are zeroed.
__global__ void gdn_gated_norm_kernel(const __nv_bfloat16* __restrict__ o_raw, const __nv_bfloat16* __restrict__ z,
                                      const __nv_bfloat16* __restrict__ norm_w, __nv_bfloat16* __restrict__ out,
                                      long rows, long valid_rows, int Dv, float eps) {
  const long row = static_cast<long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  if (row >= valid_rows) {
    for (int d = lane; d < Dv; d += 32) out[row * Dv + d] = __float2bfloat16(0.f);
    return;
  }
  float ss = 0.f;
  for (int d = lane; d < Dv; d += 32) {
    const float v = __bfloat162float(o_raw[row * Dv + d]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / Dv + eps);
  for (int d = lane; d < Dv; d += 32) {
    const float v = __bfloat162float(o_raw[row * Dv + d]);
    const float zz = __bfloat162float(z[row * Dv + d]);
    out[row * Dv + d] = __float2bfloat16(v * inv * __bfloat162float(norm_w[d]) * silu(zz));
  }
}

}  // namespace afd

// scratch: T * C bf16 (conv output). A_log / dt_bias fp32; everything else bf16. ld_*: row strides in
// elements of mixed, z, a and b, so that the four may be column ranges of one merged projection output.
extern "C" int afd_gdn_decode_ld(const void* mixed, const void* z, const void* a, const void* b, const void* conv_w,
                                 const void* A_log, const void* dt_bias, const void* norm_w, void* conv_state,
                                 void* rec_state, const void* slots, void* out, void* scratch, int T, int Hk, int Hv,
                                 int Dk, int Dv, int W, int num_slots, float eps, void* status, void* stream,
                                 long ld_mixed, long ld_z, long ld_a, long ld_b) {
  using namespace afd;
  if (T == 0) return 0;
  if (W < 2 || W > 9 || Hv % Hk != 0 || Dv > 256 || Dv % 32 != 0 || scratch == nullptr) return -1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int C = 2 * Hk * Dk + Hv * Dv;
  if (ld_mixed < C || ld_z < static_cast<long>(Hv) * Dv || ld_a < Hv || ld_b < Hv) return -3;
  auto y = static_cast<__nv_bfloat16*>(scratch);
  dim3 g1((C + 255) / 256, T);
  gdn_conv_step_kernel<<<g1, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(mixed), y,
                                           static_cast<const __nv_bfloat16*>(conv_w),
                                           static_cast<__nv_bfloat16*>(conv_state), static_cast<const int*>(slots), T,
                                           C, W, num_slots, static_cast<int*>(status), ld_mixed);
  AFD_CHECK_LAUNCH();
  dim3 g2(Hv, T);
#define LAUNCH_REC(DKK)                                                                                          \
  gdn_recurrent_kernel<DKK><<<g2, 256, 0, st>>>(                                                                 \
      y, static_cast<const __nv_bfloat16*>(z), static_cast<const __nv_bfloat16*>(a),                            \
      static_cast<const __nv_bfloat16*>(b), static_cast<const float*>(A_log), static_cast<const float*>(dt_bias), \
      static_cast<const __nv_bfloat16*>(norm_w), static_cast<float*>(rec_state), static_cast<const int*>(slots),  \
      static_cast<__nv_bfloat16*>(out), T, Hk, Hv, Dv, num_slots, eps, static_cast<int*>(status), ld_z, ld_a, ld_b)
  if (Dk == 128) LAUNCH_REC(128);
  else if (Dk == 64) LAUNCH_REC(64);
  else if (Dk == 32) LAUNCH_REC(32);
  else if (Dk == 256) LAUNCH_REC(256);
  else return -2;
#undef LAUNCH_REC
  AFD_CHECK_LAUNCH();
  return 0;
}

extern "C" int afd_gdn_decode(const void* mixed, const void* z, const void* a, const void* b, const void* conv_w,
                              const void* A_log, const void* dt_bias, const void* norm_w, void* conv_state,
                              void* rec_state, const void* slots, void* out, void* scratch, int T, int Hk, int Hv,
                              int Dk, int Dv, int W, int num_slots, float eps, void* status, void* stream) {
  return afd_gdn_decode_ld(mixed, z, a, b, conv_w, A_log, dt_bias, norm_w, conv_state, rec_state, slots, out, scratch,
                           T, Hk, Hv, Dk, Dv, W, num_slots, eps, status, stream, 2L * Hk * Dk + static_cast<long>(Hv) * Dv,
                           static_cast<long>(Hv) * Dv, Hv, Hv);
}

// Prefill of `num_seqs` sequences packed back to back (cu_seqlens int32 [num_seqs + 1], token
// rows past cu_seqlens[num_seqs] are padding and get zero output). fresh[s] != 0 starts sequence s
// from zero state. scratch: T * C bf16 (conv output) followed by T * Hv * Dv bf16 (raw outputs).
extern "C" int afd_gdn_prefill(const void* mixed, const void* z, const void* a, const void* b, const void* conv_w,
                               const void* A_log, const void* dt_bias, const void* norm_w, void* conv_state,
                               void* rec_state, const void* slots, const void* cu_seqlens, const void* fresh,
                               void* out, void* scratch, int T, int valid_T, int num_seqs, int Hk, int Hv, int Dk,
                               int Dv, int W, int num_slots, float eps, void* status, void* stream) {
  using namespace afd;
  if (T == 0) return 0;
  if (W < 2 || W > 9 || Hv % Hk != 0 || Dv > 256 || Dv % 8 != 0 || scratch == nullptr) return -1;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int C = 2 * Hk * Dk + Hv * Dv;
  auto y = static_cast<__nv_bfloat16*>(scratch);
  auto o_raw = y + static_cast<size_t>(T) * C;
  if (num_seqs > 0) {
    dim3 g1((C + 255) / 256, num_seqs);
    gdn_conv_prefill_kernel<<<g1, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(mixed), y,
                                                static_cast<const __nv_bfloat16*>(conv_w),
                                                static_cast<__nv_bfloat16*>(conv_state), static_cast<const int*>(slots),
                                                static_cast<const int*>(cu_seqlens), static_cast<const int*>(fresh), C,
                                                W, num_slots, static_cast<int*>(status));
    AFD_CHECK_LAUNCH();
    dim3 g2(Hv, num_seqs);
#define LAUNCH_PRE(DKK, RPW)                                                                                       \
  gdn_recurrent_prefill_kernel<DKK, RPW><<<g2, 256, 0, st>>>(                                                      \
      y, static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(b), static_cast<const float*>(A_log), \
      static_cast<const float*>(dt_bias), static_cast<float*>(rec_state), static_cast<const int*>(slots),           \
      static_cast<const int*>(cu_seqlens), static_cast<const int*>(fresh), o_raw, Hk, Hv, Dv, num_slots,            \
      static_cast<int*>(status))
    const int rpw = (Dv + 7) / 8;
    if (Dk == 128 && rpw <= 16) LAUNCH_PRE(128, 16);
    else if (Dk == 128) LAUNCH_PRE(128, 32);
    else if (Dk == 64 && rpw <= 16) LAUNCH_PRE(64, 16);
    else if (Dk == 64) LAUNCH_PRE(64, 32);
    else if (Dk == 32 && rpw <= 8) LAUNCH_PRE(32, 8);
    else if (Dk == 32) LAUNCH_PRE(32, 32);
    else return -2;
#undef LAUNCH_PRE
    AFD_CHECK_LAUNCH();
  }
  const long rows = static_cast<long>(T) * Hv;
  gdn_gated_norm_kernel<<<static_cast<unsigned int>((rows + 7) / 8), 256, 0, st>>>(
      o_raw, static_cast<const __nv_bfloat16*>(z), static_cast<const __nv_bfloat16*>(norm_w),
      static_cast<__nv_bfloat16*>(out), rows, static_cast<long>(valid_T) * Hv, Dv, eps);
  AFD_CHECK_LAUNCH();
  return 0;
}
