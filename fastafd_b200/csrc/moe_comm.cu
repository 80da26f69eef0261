// N2M dispatch / M2N combine over NVLink peer memory, and the expert-side grouping.
//
// Protocol (one "lane" = one micro-batch's private set of buffers and flags; a lane
// strictly alternates dispatch -> combine per layer, so buffers are never
// overwritten while a peer still reads them and no credit counters are needed):
//
//   attention GPU a                                  expert GPU e
//   ----------------------------------------------   ------------------------------------------
//   dispatch_push: (optional 1x128 FP8 quant of the
//     row), store the row into e's recv_x[a][t]
//     for every e that owns one of the token's
//     experts; store the token's top-k ids into
//     every e's recv_idx[a][t]; last CTA releases
//     n2m_flag[a] = epoch on every e            =>   eg_group: wait n2m_flag[*] >= epoch (bounded),
//                                                      count per local expert, pad to the token
//                                                      tile, assign pool rows, emit tile_info /
//                                                      row_meta
//                                                    eg_gather: recv_x rows -> expert-grouped pool
//                                                    grouped GEMM (SwiGLU) ; grouped GEMM (COMBINE):
//   ag_combine: wait m2n_flag[*] >= epoch       <=     rows stored into a's combine[k][t], last CTA
//     (bounded), y[t] = sum_k w[t,k] combine[k][t]     releases m2n_flag[e] = epoch on every a
//     in fp32, optional residual add + RMSNorm
//
// Epochs live in device memory and are advanced by the kernels themselves, so the
// whole exchange can sit inside a replayed CUDA graph. Every wait is bounded by a
// caller-given timeout in nanoseconds; on expiry the kernel records
// kStatusFlagTimeout in the status word and carries on without faulting.
//
// Reference behaviour: dispatch / combine roles of
// python/minisgl/kernel/csrc/deepgemm/deep_gemm/include/deep_gemm/impls/sm100_mega_moe_m2n.cuh
// (AG kernel :212-1265; EG pull + pool :2023-2254) and python/minisgl/moe/megamoe_m2n_afd.py:336-470.
// This design pushes instead of pulling and needs no global barrier.
#include "common.cuh"
#include "route_common.cuh"

namespace afd {

constexpr int kMaxRanks = 16;

struct DispatchArgs {
  const __nv_bfloat16* x;      // [T][H]
  const int* topk_idx;         // [T][K] global expert ids
  int T, H, K;
  int src_rank;                // this attention rank's index among attention ranks
  int num_eg, experts_per_eg;
  int fp8;                     // 1: quantise rows to e4m3 with 1x128 scales while pushing
  int recv_tokens;             // T capacity of the receive buffers
  void* peer_recv_x[kMaxRanks];        // [A][recv_tokens][H] bf16 or e4m3
  float* peer_recv_scale[kMaxRanks];   // [A][recv_tokens][H/128] (fp8)
  int* peer_recv_idx[kMaxRanks];       // [A][recv_tokens][K]
  uint32_t* peer_flag[kMaxRanks];      // &n2m_flag[src_rank] on each expert GPU
  uint32_t* epoch;
  unsigned int* done_counter;
  int* status;
  unsigned long long* trace;
};

__global__ void dispatch_push_kernel(const DispatchArgs a) {
  const int t = blockIdx.x;
  __shared__ uint32_t s_mask;
  if (threadIdx.x == 0) {
    uint32_t mask = 0;
    for (int k = 0; k < a.K; ++k) {
      const int e = a.topk_idx[static_cast<size_t>(t) * a.K + k];
      if (e >= 0) {
        const int eg = e / a.experts_per_eg;
        if (eg < a.num_eg) mask |= 1u << eg;
        else set_status(a.status, kStatusBadExtent);
      }
    }
    s_mask = mask;
  }
  if (threadIdx.x < a.K) {
    const int e = a.topk_idx[static_cast<size_t>(t) * a.K + threadIdx.x];
    for (int eg = 0; eg < a.num_eg; ++eg) {
      a.peer_recv_idx[eg][(static_cast<size_t>(a.src_rank) * a.recv_tokens + t) * a.K + threadIdx.x] = e;
    }
  }
  __syncthreads();
  const uint32_t mask = s_mask;
  const size_t dst_row = static_cast<size_t>(a.src_rank) * a.recv_tokens + t;
  const __nv_bfloat16* xr = a.x + static_cast<size_t>(t) * a.H;
  if (!a.fp8) {
    for (int i = threadIdx.x * 8; i < a.H; i += blockDim.x * 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
      for (int eg = 0; eg < a.num_eg; ++eg) {
        if (mask & (1u << eg)) {
          *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.peer_recv_x[eg]) + dst_row * a.H + i) = v;
        }
      }
    }
  } else {
    // one warp per 128-wide group: 4 elements per lane
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int groups = a.H / 128;
    for (int g = warp; g < groups; g += nw) {
      const uint2 raw = *reinterpret_cast<const uint2*>(xr + g * 128 + lane * 4);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float2 f0 = __bfloat1622float2(b2[0]), f1 = __bfloat1622float2(b2[1]);
      float amax = fmaxf(fmaxf(fabsf(f0.x), fabsf(f0.y)), fmaxf(fabsf(f1.x), fabsf(f1.y)));
      amax = warp_max(amax);
      const float scale = fmaxf(amax, 1e-10f) / 448.f;
      const float inv = 1.f / scale;
      uint32_t packed = 0;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f0.x * inv, __NV_SATFINITE, __NV_E4M3));
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f0.y * inv, __NV_SATFINITE, __NV_E4M3)) << 8;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f1.x * inv, __NV_SATFINITE, __NV_E4M3)) << 16;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f1.y * inv, __NV_SATFINITE, __NV_E4M3)) << 24;
      for (int eg = 0; eg < a.num_eg; ++eg) {
        if (mask & (1u << eg)) {
          *reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(a.peer_recv_x[eg]) + dst_row * a.H + g * 128 + lane * 4) = packed;
          if (lane == 0) a.peer_recv_scale[eg][dst_row * groups + g] = scale;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // gpu-scope fence + counter bump per CTA; only the last CTA pays the (chip-wide
    // serialised) system-scope fence before it releases the flags. The chain
    // data -> fence.gpu -> counter -> fence.sys -> flag orders every CTA's stores
    // before the flag for an acquiring peer.
    __threadfence();
    const unsigned int prev = atomicAdd(a.done_counter, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      const uint32_t e = *a.epoch;
      for (int eg = 0; eg < a.num_eg; ++eg) st_relaxed_sys(a.peer_flag[eg], e);   // ordered by the fence above
      trace_stamp(a.trace, e, 0);
      *a.epoch = e + 1;
      *a.done_counter = 0;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------------------
// Fused post-attention step of an attention rank, one CTA per token:
//   residual += attn_out ; x = RMSNorm(residual) * w        (x also kept locally for the
//   shared expert) ; logits = x . gate^T ; scoring + top-k (+ renorm) ; push the row and the
//   top-k ids into the expert GPUs ; last CTA releases the N2M flags.
// It replaces four launches (add+norm, gate GEMM, top-k, dispatch) on the decode path; the
// gate matrix (E x H) stays L2-resident, so re-reading it per token is cheap for decode-sized
// T. Reference: the fused tensor-core router python/minisgl/kernel/csrc/jit/gate_topk_fused.cu
// (which can also emit the dispatch quantisation) and the AG kernel's in-kernel gate
// (sm100_mega_moe_m2n.cuh:571-712).
// ---------------------------------------------------------------------------------------
struct RouteDispatchArgs {
  const __nv_bfloat16* attn_out;   // [T][H]
  __nv_bfloat16* residual;         // [T][H] in/out
  const __nv_bfloat16* norm_w;     // [H]
  const void* gate_w;              // [E][H] bf16 or fp32
  const float* gate_bias;          // [E] or null (selection bias, sigmoid scoring)
  __nv_bfloat16* x_out;            // [T][H] normed hidden (local copy)
  int* topk_idx_out;               // [T][K]
  float* topk_w_out;               // [T][K]
  int E, gate_fp32, scoring, renorm, offset1;
  int mma_logits;                  // bf16 gate, shapes that the tensor-core GEMV covers
  float eps, route_scale;
  DispatchArgs d;                  // d.x / d.topk_idx are ignored (produced here)
};

__global__ void __launch_bounds__(1024) ag_route_dispatch_kernel(const RouteDispatchArgs a) {
  // shared: x as bf16 (H * 2 bytes, 16-byte aligned rows read as uint4: conflict-free) |
  //         logits (E floats) | red (32 floats)
  extern __shared__ __align__(16) uint8_t rsm_raw[];
  const DispatchArgs& d = a.d;
  const int H = d.H, t = blockIdx.x;
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(rsm_raw);
  float* s_logit = reinterpret_cast<float*>(rsm_raw + static_cast<size_t>(H) * 2);
  float* red = s_logit + a.E;
  float* s_part = red + 32;        // [nsplit][ET*16] partial logits of the tensor-core GEMV
  __shared__ int s_idx[32];
  __shared__ float s_w[32];
  __shared__ uint32_t s_mask;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;

  // 0. pull the gate matrix towards L2 while the norm runs: it was last touched a whole
  //    decode step ago, and the logits loop below is a chain of dependent loads.
  {
    const size_t gate_bytes = static_cast<size_t>(a.E) * H * (a.gate_fp32 ? 4 : 2);
    const char* gp = static_cast<const char*>(a.gate_w);
    const size_t per_cta = (gate_bytes / gridDim.x + 127) / 128 * 128;
    const size_t lo = per_cta * blockIdx.x, hi = min(gate_bytes, lo + per_cta);
    for (size_t off = lo + static_cast<size_t>(threadIdx.x) * 128; off < hi; off += static_cast<size_t>(blockDim.x) * 128) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(gp + off));
    }
  }

  // 1. residual add + RMSNorm (each thread keeps its 8 elements in registers; H <= 8 * 1024)
  float rv8[8];
  float ss = 0.f;
  const int i0 = threadIdx.x * 8;
  const bool active = i0 < H;
  if (active) {
    const uint4 xa = *reinterpret_cast<const uint4*>(a.attn_out + static_cast<size_t>(t) * H + i0);
    uint4 ra = *reinterpret_cast<const uint4*>(a.residual + static_cast<size_t>(t) * H + i0);
    const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xa);
    __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&ra);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 xv = __bfloat1622float2(x2[j]);
      float2 rv = __bfloat1622float2(r2[j]);
      rv.x += xv.x;
      rv.y += xv.y;
      r2[j] = __floats2bfloat162_rn(rv.x, rv.y);
      rv = __bfloat1622float2(r2[j]);
      rv8[2 * j] = rv.x;
      rv8[2 * j + 1] = rv.y;
      ss += rv.x * rv.x + rv.y * rv.y;
    }
    *reinterpret_cast<uint4*>(a.residual + static_cast<size_t>(t) * H + i0) = ra;
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = lane < nw ? red[lane] : 0.f;
  tot = warp_sum(tot);
  const float inv = rsqrtf(tot / H + a.eps);
  if (active) {
    const uint4 wa = *reinterpret_cast<const uint4*>(a.norm_w + i0);
    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wa);
    uint4 oa;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&oa);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 g = __bfloat1622float2(w2[j]);
      if (a.offset1) {
        g.x += 1.f;
        g.y += 1.f;
      }
      o2[j] = __floats2bfloat162_rn(rv8[2 * j] * inv * g.x, rv8[2 * j + 1] * inv * g.y);
    }
    *reinterpret_cast<uint4*>(a.x_out + static_cast<size_t>(t) * H + i0) = oa;
    *reinterpret_cast<uint4*>(xs + i0) = oa;          // the router sees the bf16-rounded x
  }
  __syncthreads();

  // 2. router logits: one warp per expert, lanes split H. CTAs start at different experts so
  //    that they do not all pull the same gate rows out of L2 at the same moment.
  const int rot = (blockIdx.x * 5) % a.E;
  if (a.gate_fp32) {
    for (int e0 = warp; e0 < a.E; e0 += nw) {
      int e = e0 + rot;
      if (e >= a.E) e -= a.E;
      float acc = 0.f;
      const float* g = static_cast<const float*>(a.gate_w) + static_cast<size_t>(e) * H;
#pragma unroll 4
      for (int i = lane * 8; i < H; i += 256) {
        const float4 g0 = *reinterpret_cast<const float4*>(g + i);
        const float4 g1 = *reinterpret_cast<const float4*>(g + i + 4);
        const uint4 xa = *reinterpret_cast<const uint4*>(xs + i);
        const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xa);
        const float2 a0 = __bfloat1622float2(x2[0]), a1 = __bfloat1622float2(x2[1]);
        const float2 a2 = __bfloat1622float2(x2[2]), a3 = __bfloat1622float2(x2[3]);
        acc += g0.x * a0.x + g0.y * a0.y + g0.z * a1.x + g0.w * a1.y + g1.x * a2.x + g1.y * a2.y + g1.z * a3.x + g1.w * a3.y;
      }
      acc = warp_sum(acc);
      if (lane == 0) s_logit[e] = acc;
    }
  } else if (a.mma_logits) {
    // Tensor-core GEMV: a warp owns 16 experts (the MMA M side) over one slice of H; the token is
    // the B operand (all 8 columns carry the same x, column 0 is read back). A lane loads 16
    // contiguous bytes of two gate rows per 32 columns and feeds two m16n8k16 MMAs with them: the
    // columns are consumed in a permuted order, the same for both operands, which a dot product
    // does not see. ~25x fewer issued instructions than the FMA loop; bound by the L2 read.
    const int ET = (a.E + 15) >> 4;                 // expert tiles
    const int nsplit = max(1, nw / ET);             // K slices (a power of two for ET 8/16/32)
    const int g = lane >> 2, t4 = lane & 3;
    for (int job = warp; job < ET * nsplit; job += nw) {
      int et = job % ET + (blockIdx.x % ET);        // CTAs start at different expert tiles
      if (et >= ET) et -= ET;
      const int ks = job / ET;
      const int kb0 = ks * (H / 32 / nsplit), kb1 = kb0 + H / 32 / nsplit;
      const int r_lo = min(et * 16 + g, a.E - 1), r_hi = min(et * 16 + g + 8, a.E - 1);
      const __nv_bfloat16* g_lo = static_cast<const __nv_bfloat16*>(a.gate_w) + static_cast<size_t>(r_lo) * H + t4 * 8;
      const __nv_bfloat16* g_hi = static_cast<const __nv_bfloat16*>(a.gate_w) + static_cast<size_t>(r_hi) * H + t4 * 8;
      float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int kb = kb0; kb < kb1; kb += 2) {      // the slice is a whole number of pairs (host check)
        uint4 lo[2], hi[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          lo[u] = *reinterpret_cast<const uint4*>(g_lo + (kb + u) * 32);
          hi[u] = *reinterpret_cast<const uint4*>(g_hi + (kb + u) * 32);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + (kb + u) * 32 + t4 * 8);
            mma_gemv_16816(c, lo[u].x, hi[u].x, lo[u].y, hi[u].y, xv.x, xv.y);
            mma_gemv_16816(c, lo[u].z, hi[u].z, lo[u].w, hi[u].w, xv.z, xv.w);
          }
        }
      }
      if (t4 == 0) {
        float* part = s_part + ks * (ET * 16);
        part[et * 16 + g] = c[0];
        part[et * 16 + g + 8] = c[2];
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < a.E; e += blockDim.x) {
      float v = 0.f;
      for (int ks = 0; ks < nsplit; ++ks) v += s_part[ks * (ET * 16) + e];
      s_logit[e] = v;
    }
  } else {
    // two experts per pass, every load of both rows issued before the first use
    const int iters = H / 256;            // <= 16
    for (int e0 = warp; e0 < a.E; e0 += 2 * nw) {
      int ea = e0 + rot, eb = e0 + nw + rot;
      if (ea >= a.E) ea -= a.E;
      const bool has_b = e0 + nw < a.E;
      if (eb >= a.E) eb -= a.E;
      if (!has_b) eb = ea;
      const __nv_bfloat16* ga = static_cast<const __nv_bfloat16*>(a.gate_w) + static_cast<size_t>(ea) * H;
      const __nv_bfloat16* gb = static_cast<const __nv_bfloat16*>(a.gate_w) + static_cast<size_t>(eb) * H;
      float acc_a = 0.f, acc_b = 0.f;
#pragma unroll 1
      for (int base = 0; base < iters; base += 4) {
        uint4 ba[4], bb[4];
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          if (base + it < iters) {
            ba[it] = *reinterpret_cast<const uint4*>(ga + (base + it) * 256 + lane * 8);
            bb[it] = *reinterpret_cast<const uint4*>(gb + (base + it) * 256 + lane * 8);
          }
        }
#pragma unroll
        for (int it = 0; it < 4; ++it) {
          if (base + it < iters) {
            const uint4 xa = *reinterpret_cast<const uint4*>(xs + (base + it) * 256 + lane * 8);
            const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xa);
            const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&ba[it]);
            const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&bb[it]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 xv = __bfloat1622float2(x2[j]);
              const float2 av = __bfloat1622float2(a2[j]);
              const float2 bv = __bfloat1622float2(b2[j]);
              acc_a = fmaf(av.x, xv.x, acc_a);
              acc_a = fmaf(av.y, xv.y, acc_a);
              acc_b = fmaf(bv.x, xv.x, acc_b);
              acc_b = fmaf(bv.y, xv.y, acc_b);
            }
          }
        }
      }
      acc_a = warp_sum(acc_a);
      acc_b = warp_sum(acc_b);
      if (lane == 0) {
        s_logit[ea] = acc_a;
        if (has_b) s_logit[eb] = acc_b;
      }
    }
  }
  __syncthreads();

  // 3. scoring + top-k by warp 0
  if (warp == 0) {
    if (a.E <= 128) warp_topk<4>(s_logit, a.gate_bias, a.E, d.K, a.scoring, a.renorm, a.route_scale, s_idx, s_w, lane);
    else if (a.E <= 256) warp_topk<8>(s_logit, a.gate_bias, a.E, d.K, a.scoring, a.renorm, a.route_scale, s_idx, s_w, lane);
    else warp_topk<16>(s_logit, a.gate_bias, a.E, d.K, a.scoring, a.renorm, a.route_scale, s_idx, s_w, lane);
    __syncwarp();
    uint32_t mask = 0;
    if (lane < d.K) {
      const int e = s_idx[lane];
      a.topk_idx_out[static_cast<size_t>(t) * d.K + lane] = e;
      a.topk_w_out[static_cast<size_t>(t) * d.K + lane] = s_w[lane];
      const int eg = e / d.experts_per_eg;
      if (eg < d.num_eg) mask = 1u << eg;
      else set_status(d.status, kStatusBadExtent);
      for (int g = 0; g < d.num_eg; ++g) {
        d.peer_recv_idx[g][(static_cast<size_t>(d.src_rank) * d.recv_tokens + t) * d.K + lane] = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mask |= __shfl_xor_sync(0xffffffffu, mask, o);
    if (lane == 0) s_mask = mask;
  }
  __syncthreads();

  // 4. push the row to every expert GPU that owns one of its experts
  const uint32_t mask = s_mask;
  const size_t dst_row = static_cast<size_t>(d.src_rank) * d.recv_tokens + t;
  if (!d.fp8) {
    for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(xs + i);
      for (int g = 0; g < d.num_eg; ++g) {
        if (mask & (1u << g)) {
          *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(d.peer_recv_x[g]) + dst_row * H + i) = v;
        }
      }
    }
  } else {
    const int groups = H / 128;
    for (int g128 = warp; g128 < groups; g128 += nw) {
      const uint2 fr = *reinterpret_cast<const uint2*>(xs + g128 * 128 + lane * 4);
      const __nv_bfloat162* f2 = reinterpret_cast<const __nv_bfloat162*>(&fr);
      const float2 fa = __bfloat1622float2(f2[0]), fb = __bfloat1622float2(f2[1]);
      const float4 f = make_float4(fa.x, fa.y, fb.x, fb.y);
      float amax = fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w)));
      amax = warp_max(amax);
      const float scale = fmaxf(amax, 1e-10f) / 448.f;
      const float is = 1.f / scale;
      uint32_t packed = 0;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f.x * is, __NV_SATFINITE, __NV_E4M3));
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f.y * is, __NV_SATFINITE, __NV_E4M3)) << 8;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f.z * is, __NV_SATFINITE, __NV_E4M3)) << 16;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f.w * is, __NV_SATFINITE, __NV_E4M3)) << 24;
      for (int g = 0; g < d.num_eg; ++g) {
        if (mask & (1u << g)) {
          *reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(d.peer_recv_x[g]) + dst_row * H + g128 * 128 + lane * 4) = packed;
          if (lane == 0) d.peer_recv_scale[g][dst_row * groups + g128] = scale;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();              // see dispatch_push_kernel: one system fence, by the last CTA
    const unsigned int prev = atomicAdd(d.done_counter, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      const uint32_t e = *d.epoch;
      for (int g = 0; g < d.num_eg; ++g) st_relaxed_sys(d.peer_flag[g], e);   // ordered by the fence above
      trace_stamp(d.trace, e, 0);
      *d.epoch = e + 1;
      *d.done_counter = 0;
      __threadfence();
    }
  }
}

struct GroupArgs {
  const int* recv_idx;       // [A][recv_tokens][K]
  const uint32_t* n2m_flag;  // [A]
  uint32_t* epoch;           // expected epoch, advanced by the kernel
  int A, T, K, recv_tokens;
  int expert_base, experts_local;
  int block_tok;
  int pool_rows, max_tok_tiles;
  uint32_t* row_meta;        // [pool_rows]
  int4* tile_info;           // [max_tok_tiles]
  int* counters;             // [0] = num_tok_tiles, [1] = total rows (padded), [2] = routed rows
  int* expert_counts;        // [experts_local] (for load statistics), may be null
  uint64_t timeout_ns;
  int* status;
  unsigned long long* trace;
};

// One CTA. Shared memory: 3 * experts_local ints.
__global__ void eg_group_kernel(const GroupArgs a) {
  extern __shared__ int sm[];
  int* cnt = sm;
  int* off = sm + a.experts_local;
  int* cur = sm + 2 * a.experts_local;
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) {
    s_epoch = *a.epoch;
    trace_stamp(a.trace, s_epoch, 0);
  }
  for (int e = threadIdx.x; e < a.experts_local; e += blockDim.x) {
    cnt[e] = 0;
    cur[e] = 0;
  }
  __syncthreads();
  if (threadIdx.x < a.A) wait_flag_ge(a.n2m_flag + threadIdx.x, s_epoch, a.timeout_ns, a.status);
  __syncthreads();
  if (threadIdx.x == 0) trace_stamp(a.trace, s_epoch, 1);
  const int per_src = a.T * a.K;
  const int total = a.A * per_src;
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int src = i / per_src, r = i - src * per_src;
    const int e = a.recv_idx[static_cast<size_t>(src) * a.recv_tokens * a.K + r] - a.expert_base;
    if (e >= 0 && e < a.experts_local) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // Exclusive scan over the local experts of (token tiles, padded rows): one thread per
  // expert, chunks of 1024 experts at a time, shuffle scan inside warps + a scan of warp sums.
  {
    __shared__ int s_wtiles[32], s_wrouted[32];
    __shared__ int s_base_tiles, s_base_routed;
    if (threadIdx.x == 0) {
      s_base_tiles = 0;
      s_base_routed = 0;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int e0 = 0; e0 < a.experts_local; e0 += blockDim.x) {
      const int e = e0 + threadIdx.x;
      const int c = e < a.experts_local ? cnt[e] : 0;
      const int nt = (c + a.block_tok - 1) / a.block_tok;
      int incl_t = nt, incl_c = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int vt = __shfl_up_sync(0xffffffffu, incl_t, o);
        const int vc = __shfl_up_sync(0xffffffffu, incl_c, o);
        if (lane >= o) {
          incl_t += vt;
          incl_c += vc;
        }
      }
      if (lane == 31) {
        s_wtiles[warp] = incl_t;
        s_wrouted[warp] = incl_c;
      }
      __syncthreads();
      if (warp == 0) {
        int wt = lane < (blockDim.x >> 5) ? s_wtiles[lane] : 0;
        int wc = lane < (blockDim.x >> 5) ? s_wrouted[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int vt = __shfl_up_sync(0xffffffffu, wt, o);
          const int vc = __shfl_up_sync(0xffffffffu, wc, o);
          if (lane >= o) {
            wt += vt;
            wc += vc;
          }
        }
        s_wtiles[lane] = wt;       // inclusive sums of the warps
        s_wrouted[lane] = wc;
      }
      __syncthreads();
      const int warp_off_t = warp > 0 ? s_wtiles[warp - 1] : 0;
      const int tile0 = s_base_tiles + warp_off_t + incl_t - nt;     // first tile of expert e
      if (e < a.experts_local) {
        off[e] = tile0 * a.block_tok;
        for (int j = 0; j < nt; ++j) {
          if (tile0 + j < a.max_tok_tiles) {
            a.tile_info[tile0 + j] =
                make_int4(e, (tile0 + j) * a.block_tok, min(a.block_tok, c - j * a.block_tok), 0);
          }
        }
        if (a.expert_counts) a.expert_counts[e] = c;
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        s_base_tiles += s_wtiles[(blockDim.x >> 5) - 1];
        s_base_routed += s_wrouted[(blockDim.x >> 5) - 1];
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      int tiles = s_base_tiles;
      const int rows = tiles * a.block_tok;
      if (tiles > a.max_tok_tiles || rows > a.pool_rows) {
        set_status(a.status, kStatusCapacity);
        tiles = min(tiles, a.max_tok_tiles);
      }
      a.counters[0] = tiles;
      a.counters[1] = rows;
      a.counters[2] = s_base_routed;
      *a.epoch = s_epoch + 1;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < total; i += blockDim.x) {
    const int src = i / per_src, r = i - src * per_src;
    const int t = r / a.K, k = r - t * a.K;
    const int e = a.recv_idx[static_cast<size_t>(src) * a.recv_tokens * a.K + r] - a.expert_base;
    if (e >= 0 && e < a.experts_local) {
      const int row = off[e] + atomicAdd(&cur[e], 1);
      if (row < a.pool_rows) {
        a.row_meta[row] = (static_cast<uint32_t>(src) << 24) | (static_cast<uint32_t>(k) << 16) |
                          static_cast<uint32_t>(t);
      }
    }
  }
  // mark padding rows (never read by the combine epilogue: valid_rows excludes them)
}

struct GatherArgs {
  const void* recv_x;          // [A][recv_tokens][H]
  const float* recv_scale;     // fp8: [A][recv_tokens][H/128]
  const uint32_t* row_meta;
  const int4* tile_info;
  const int* counters;
  void* pool_x;                // [pool_rows][H]
  float* pool_scale;           // fp8: [pool_rows][H/128]
  int recv_tokens, row_bytes, scale_per_row, block_tok, max_tok_tiles;
};

// One CTA per (token tile); copies the tile's valid rows into the pool.
__global__ void eg_gather_kernel(const GatherArgs a) {
  const int ntiles = min(a.counters[0], a.max_tok_tiles);
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int4 ti = a.tile_info[tile];
    const int vec_per_row = a.row_bytes / 16;
    for (int idx = threadIdx.x; idx < ti.z * vec_per_row; idx += blockDim.x) {
      const int r = idx / vec_per_row, v = idx - r * vec_per_row;
      const int row = ti.y + r;
      const uint32_t meta = a.row_meta[row];
      const int src = meta >> 24, tok = meta & 0xffff;
      const uint4* s = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.recv_x) +
                                                      (static_cast<size_t>(src) * a.recv_tokens + tok) * a.row_bytes);
      reinterpret_cast<uint4*>(static_cast<uint8_t*>(a.pool_x) + static_cast<size_t>(row) * a.row_bytes)[v] = s[v];
    }
    if (a.recv_scale != nullptr) {
      for (int idx = threadIdx.x; idx < ti.z * a.scale_per_row; idx += blockDim.x) {
        const int r = idx / a.scale_per_row, v = idx - r * a.scale_per_row;
        const int row = ti.y + r;
        const uint32_t meta = a.row_meta[row];
        const int src = meta >> 24, tok = meta & 0xffff;
        a.pool_scale[static_cast<size_t>(row) * a.scale_per_row + v] =
            a.recv_scale[(static_cast<size_t>(src) * a.recv_tokens + tok) * a.scale_per_row + v];
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// Decode-sized grouping + gather in ONE launch (no single-CTA stage, no second launch):
// CTA j owns token tile j. Every CTA waits for the attention ranks' flags itself, rebuilds
// the per-expert histogram from the received top-k ids (a few KB), finds the expert and
// row range of its tile, selects its rows in entry order (deterministic: all CTAs agree
// without talking to each other), writes tile_info[j] / row_meta and copies the rows into
// the expert-grouped pool. Used when A*T*K <= kFusedGroupMaxEntries.
// ---------------------------------------------------------------------------------------
constexpr int kFusedGroupMaxEntries = 8192;
constexpr int kFusedGroupThreads = 256;

struct FusedGroupArgs {
  GroupArgs g;
  const void* recv_x;
  const float* recv_scale;
  void* pool_x;
  float* pool_scale;
  int row_bytes, scale_per_row;
  unsigned int* done_counter;
};

__global__ void __launch_bounds__(kFusedGroupThreads) eg_group_gather_fused_kernel(const FusedGroupArgs fa) {
  const GroupArgs& a = fa.g;
  extern __shared__ int sm[];
  int* cnt = sm;                              // [experts_local]
  int* tstart = sm + a.experts_local;         // [experts_local + 1] first tile of each expert
  __shared__ uint32_t s_epoch;
  __shared__ int s_e, s_first, s_total_tiles, s_routed;
  __shared__ int s_wsum[kFusedGroupThreads / 32];
  __shared__ uint32_t s_meta[128];            // rows of this tile (block_tok <= 128)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    s_epoch = *a.epoch;
    s_e = -1;
    if (blockIdx.x == 0) trace_stamp(a.trace, s_epoch, 0);
  }
  for (int e = tid; e < a.experts_local; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  if (tid < a.A) wait_flag_ge(a.n2m_flag + tid, s_epoch, a.timeout_ns, a.status);
  __syncthreads();
  if (tid == 0 && blockIdx.x == 0) trace_stamp(a.trace, s_epoch, 1);

  const int per_src = a.T * a.K;
  const int total = a.A * per_src;
  // histogram over all entries
  for (int i = tid; i < total; i += blockDim.x) {
    const int src = i / per_src, r = i - src * per_src;
    const int e = a.recv_idx[static_cast<size_t>(src) * a.recv_tokens * a.K + r] - a.expert_base;
    if (e >= 0 && e < a.experts_local) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  // tile prefix over experts: warp 0, each lane a contiguous slice of experts
  if (warp == 0) {
    const int per = (a.experts_local + 31) / 32;
    const int lo = min(lane * per, a.experts_local), hi = min(lo + per, a.experts_local);
    int t = 0, c = 0;
    for (int e = lo; e < hi; ++e) {
      t += (cnt[e] + a.block_tok - 1) / a.block_tok;
      c += cnt[e];
    }
    int incl = t, cincl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      const int vc = __shfl_up_sync(0xffffffffu, cincl, o);
      if (lane >= o) {
        incl += v;
        cincl += vc;
      }
    }
    int run = incl - t;
    for (int e = lo; e < hi; ++e) {
      tstart[e] = run;
      run += (cnt[e] + a.block_tok - 1) / a.block_tok;
    }
    if (lane == 31) {
      tstart[a.experts_local] = incl;
      s_total_tiles = incl;
      s_routed = cincl;
    }
  }
  __syncthreads();
  const int my_tile = blockIdx.x;
  for (int e = tid; e < a.experts_local; e += blockDim.x) {
    if (tstart[e] <= my_tile && my_tile < tstart[e + 1]) {
      s_e = e;
      s_first = my_tile - tstart[e];
    }
  }
  __syncthreads();
  const int e_mine = s_e;
  if (e_mine >= 0) {
    const int want_lo = s_first * a.block_tok;
    const int valid = min(a.block_tok, cnt[e_mine] - want_lo);
    const int row0 = my_tile * a.block_tok;
    // ordered rank of every matching entry: contiguous chunk per thread + block scan
    const int per = (total + blockDim.x - 1) / blockDim.x;
    const int lo = min(tid * per, total), hi = min(lo + per, total);
    int mine = 0;
    for (int i = lo; i < hi; ++i) {
      const int src = i / per_src, r = i - src * per_src;
      mine += (a.recv_idx[static_cast<size_t>(src) * a.recv_tokens * a.K + r] - a.expert_base) == e_mine;
    }
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) s_wsum[warp] = incl;
    __syncthreads();
    int base = incl - mine;
    for (int w = 0; w < warp; ++w) base += s_wsum[w];
    for (int i = lo; i < hi; ++i) {
      const int src = i / per_src, r = i - src * per_src;
      if ((a.recv_idx[static_cast<size_t>(src) * a.recv_tokens * a.K + r] - a.expert_base) == e_mine) {
        const int slot = base - want_lo;
        if (slot >= 0 && slot < valid) {
          const int t = r / a.K, k = r - t * a.K;
          s_meta[slot] = (static_cast<uint32_t>(src) << 24) | (static_cast<uint32_t>(k) << 16) | static_cast<uint32_t>(t);
        }
        ++base;
      }
    }
    __syncthreads();
    if (row0 + a.block_tok <= a.pool_rows && my_tile < a.max_tok_tiles) {
      if (tid == 0) a.tile_info[my_tile] = make_int4(e_mine, row0, valid, 0);
      for (int i = tid; i < valid; i += blockDim.x) a.row_meta[row0 + i] = s_meta[i];
      const int vec_per_row = fa.row_bytes / 16;
      for (int idx = tid; idx < valid * vec_per_row; idx += blockDim.x) {
        const int r = idx / vec_per_row, v = idx - r * vec_per_row;
        const uint32_t meta = s_meta[r];
        const int src = meta >> 24, tok = meta & 0xffff;
        const uint4* sp = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(fa.recv_x) +
                                                         (static_cast<size_t>(src) * a.recv_tokens + tok) * fa.row_bytes);
        reinterpret_cast<uint4*>(static_cast<uint8_t*>(fa.pool_x) + static_cast<size_t>(row0 + r) * fa.row_bytes)[v] = sp[v];
      }
      if (fa.recv_scale != nullptr) {
        for (int idx = tid; idx < valid * fa.scale_per_row; idx += blockDim.x) {
          const int r = idx / fa.scale_per_row, v = idx - r * fa.scale_per_row;
          const uint32_t meta = s_meta[r];
          const int src = meta >> 24, tok = meta & 0xffff;
          fa.pool_scale[static_cast<size_t>(row0 + r) * fa.scale_per_row + v] =
              fa.recv_scale[(static_cast<size_t>(src) * a.recv_tokens + tok) * fa.scale_per_row + v];
        }
      }
    } else {
      set_status(a.status, kStatusCapacity);
    }
  }
  if (blockIdx.x == 0) {
    for (int e = tid; e < a.experts_local; e += blockDim.x) {
      if (a.expert_counts) a.expert_counts[e] = cnt[e];
    }
    if (tid == 0) {
      int tiles = s_total_tiles;
      if (tiles > a.max_tok_tiles || tiles > static_cast<int>(gridDim.x) || tiles * a.block_tok > a.pool_rows) {
        set_status(a.status, kStatusCapacity);
        tiles = min(min(tiles, a.max_tok_tiles), static_cast<int>(gridDim.x));
      }
      a.counters[0] = tiles;
      a.counters[1] = tiles * a.block_tok;
      a.counters[2] = s_routed;
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(fa.done_counter, 1u);
    if (prev == gridDim.x - 1) {
      trace_stamp(a.trace, s_epoch, 2);
      *a.epoch = s_epoch + 1;
      *fa.done_counter = 0;
      __threadfence();
    }
  }
}

struct CombineArgs {
  const __nv_bfloat16* combine;   // [K][combine_tokens][H]
  const float* topk_w;            // [T][K]
  const int* topk_idx;            // [T][K] (entries < 0 are skipped)
  const uint32_t* m2n_flag;       // [num_eg]
  uint32_t* epoch;
  unsigned int* done_counter;
  int T, H, K, combine_tokens, num_eg;
  float scale;                    // routed_scaling_factor
  const __nv_bfloat16* extra;     // optional [T][H] added to y (shared-expert output)
  __nv_bfloat16* y;               // [T][H] (may be null when norm outputs are given)
  // optional fused residual add + RMSNorm of the next block
  __nv_bfloat16* residual;        // [T][H] in/out
  const __nv_bfloat16* norm_w;    // [H]
  __nv_bfloat16* normed;          // [T][H]
  float eps;
  int offset1;
  uint64_t timeout_ns;
  int* status;
  unsigned long long* trace;
};

__global__ void ag_combine_kernel(const CombineArgs a) {
  extern __shared__ float sbuf[];   // H floats + 32
  float* red = sbuf + a.H;
  __shared__ uint32_t s_epoch;
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) {
    s_epoch = *a.epoch;
    if (blockIdx.x == 0) trace_stamp(a.trace, s_epoch, 1);
  }
  __syncthreads();
  if (threadIdx.x < a.num_eg) wait_flag_ge(a.m2n_flag + threadIdx.x, s_epoch, a.timeout_ns, a.status);
  __syncthreads();
  if (threadIdx.x == 0 && blockIdx.x == 0) trace_stamp(a.trace, s_epoch, 2);
  const int t = blockIdx.x;
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < a.H; i += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < a.K; ++k) {
      if (a.topk_idx != nullptr && a.topk_idx[static_cast<size_t>(t) * a.K + k] < 0) continue;
      const float w = a.topk_w[static_cast<size_t>(t) * a.K + k];
      const uint4 raw = *reinterpret_cast<const uint4*>(
          a.combine + (static_cast<size_t>(k) * a.combine_tokens + t) * a.H + i);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(b2[j]);
        acc[2 * j] = fmaf(w, f.x, acc[2 * j]);
        acc[2 * j + 1] = fmaf(w, f.y, acc[2 * j + 1]);
      }
    }
    uint4 oraw;
    __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&oraw);
    uint4 eraw = make_uint4(0, 0, 0, 0);
    if (a.extra) eraw = *reinterpret_cast<const uint4*>(a.extra + static_cast<size_t>(t) * a.H + i);
    const __nv_bfloat162* e2 = reinterpret_cast<const __nv_bfloat162*>(&eraw);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float vx = acc[2 * j] * a.scale, vy = acc[2 * j + 1] * a.scale;
      if (a.extra) {
        const float2 f = __bfloat1622float2(e2[j]);
        vx += f.x;
        vy += f.y;
      }
      o2[j] = __floats2bfloat162_rn(vx, vy);
    }
    if (a.y) *reinterpret_cast<uint4*>(a.y + static_cast<size_t>(t) * a.H + i) = oraw;
    if (a.residual) {
      uint4 rraw = *reinterpret_cast<const uint4*>(a.residual + static_cast<size_t>(t) * a.H + i);
      __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&rraw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 yv = __bfloat1622float2(o2[j]);
        float2 rv = __bfloat1622float2(r2[j]);
        rv.x += yv.x;
        rv.y += yv.y;
        r2[j] = __floats2bfloat162_rn(rv.x, rv.y);
        rv = __bfloat1622float2(r2[j]);
        sbuf[i + 2 * j] = rv.x;
        sbuf[i + 2 * j + 1] = rv.y;
        ss += rv.x * rv.x + rv.y * rv.y;
      }
      *reinterpret_cast<uint4*>(a.residual + static_cast<size_t>(t) * a.H + i) = rraw;
    }
  }
  if (a.residual && a.normed) {
    ss = warp_sum(ss);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = lane < (blockDim.x >> 5) ? red[lane] : 0.f;
    tot = warp_sum(tot);
    const float inv = rsqrtf(tot / a.H + a.eps);
    for (int i = threadIdx.x * 8; i < a.H; i += blockDim.x * 8) {
      const uint4 wraw = *reinterpret_cast<const uint4*>(a.norm_w + i);
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wraw);
      uint4 oraw;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&oraw);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 g = __bfloat1622float2(w2[j]);
        if (a.offset1) {
          g.x += 1.f;
          g.y += 1.f;
        }
        o2[j] = __floats2bfloat162_rn(sbuf[i + 2 * j] * inv * g.x, sbuf[i + 2 * j + 1] * inv * g.y);
      }
      *reinterpret_cast<uint4*>(a.normed + static_cast<size_t>(t) * a.H + i) = oraw;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(a.done_counter, 1u);
    if (prev == gridDim.x - 1) {
      trace_stamp(a.trace, s_epoch, 3);
      *a.epoch = s_epoch + 1;
      *a.done_counter = 0;
      __threadfence();
    }
  }
}

// A bounded wait on one flag as a kernel of its own: used by tests (a flag that
// nothing sets must come back as a timeout status, with the context intact) and
// by the host runtime to order a stream after a peer's signal.
__global__ void wait_flag_kernel(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, int* status) {
  if (threadIdx.x == 0) wait_flag_ge(flag, target, timeout_ns, status);
}
__global__ void set_flag_kernel(uint32_t* flag, uint32_t value) {
  if (threadIdx.x == 0) {
    __threadfence_system();
    st_release_sys(flag, value);
  }
}

}  // namespace afd

using namespace afd;

struct AfdDispatchDesc {
  const void* x; const void* topk_idx;
  int T, H, K, src_rank, num_eg, experts_per_eg, fp8, recv_tokens;
  void* peer_recv_x[kMaxRanks]; void* peer_recv_scale[kMaxRanks]; void* peer_recv_idx[kMaxRanks];
  void* peer_flag[kMaxRanks];
  void* epoch; void* done_counter; void* status; void* trace;
};

extern "C" int afd_dispatch_push(const AfdDispatchDesc* d, void* stream) {
  if (d->T == 0) return -1;   // a lane always pushes at least its padding tokens
  if (d->num_eg > kMaxRanks || d->H % 128 != 0 || d->K > 32 || d->T > d->recv_tokens) return -2;
  DispatchArgs a{};
  a.x = static_cast<const __nv_bfloat16*>(d->x);
  a.topk_idx = static_cast<const int*>(d->topk_idx);
  a.T = d->T; a.H = d->H; a.K = d->K; a.src_rank = d->src_rank; a.num_eg = d->num_eg;
  a.experts_per_eg = d->experts_per_eg; a.fp8 = d->fp8; a.recv_tokens = d->recv_tokens;
  for (int i = 0; i < d->num_eg; ++i) {
    a.peer_recv_x[i] = d->peer_recv_x[i];
    a.peer_recv_scale[i] = static_cast<float*>(d->peer_recv_scale[i]);
    a.peer_recv_idx[i] = static_cast<int*>(d->peer_recv_idx[i]);
    a.peer_flag[i] = static_cast<uint32_t*>(d->peer_flag[i]);
  }
  a.epoch = static_cast<uint32_t*>(d->epoch);
  a.done_counter = static_cast<unsigned int*>(d->done_counter);
  a.status = static_cast<int*>(d->status);
  a.trace = static_cast<unsigned long long*>(d->trace);
  dispatch_push_kernel<<<d->T, 256, 0, static_cast<cudaStream_t>(stream)>>>(a);
  AFD_CHECK_LAUNCH();
  return 0;
}

struct AfdRouteDispatchDesc {
  const void* attn_out; void* residual; const void* norm_w; const void* gate_w; const void* gate_bias;
  void* x_out; void* topk_idx_out; void* topk_w_out;
  int E, gate_fp32, scoring, renorm, offset1;
  float eps, route_scale;
  AfdDispatchDesc d;
};

extern "C" int afd_ag_route_dispatch(const AfdRouteDispatchDesc* r, void* stream) {
  const AfdDispatchDesc* d = &r->d;
  if (d->T == 0) return -1;
  if (d->num_eg > kMaxRanks || d->H % 256 != 0 || d->H > 4096 || d->K > 32 || d->T > d->recv_tokens || r->E > 512) return -2;
  RouteDispatchArgs a{};
  a.attn_out = static_cast<const __nv_bfloat16*>(r->attn_out);
  a.residual = static_cast<__nv_bfloat16*>(r->residual);
  a.norm_w = static_cast<const __nv_bfloat16*>(r->norm_w);
  a.gate_w = r->gate_w;
  a.gate_bias = static_cast<const float*>(r->gate_bias);
  a.x_out = static_cast<__nv_bfloat16*>(r->x_out);
  a.topk_idx_out = static_cast<int*>(r->topk_idx_out);
  a.topk_w_out = static_cast<float*>(r->topk_w_out);
  a.E = r->E; a.gate_fp32 = r->gate_fp32; a.scoring = r->scoring; a.renorm = r->renorm; a.offset1 = r->offset1;
  a.eps = r->eps; a.route_scale = r->route_scale;
  DispatchArgs& da = a.d;
  da.T = d->T; da.H = d->H; da.K = d->K; da.src_rank = d->src_rank; da.num_eg = d->num_eg;
  da.experts_per_eg = d->experts_per_eg; da.fp8 = d->fp8; da.recv_tokens = d->recv_tokens;
  for (int i = 0; i < d->num_eg; ++i) {
    da.peer_recv_x[i] = d->peer_recv_x[i];
    da.peer_recv_scale[i] = static_cast<float*>(d->peer_recv_scale[i]);
    da.peer_recv_idx[i] = static_cast<int*>(d->peer_recv_idx[i]);
    da.peer_flag[i] = static_cast<uint32_t*>(d->peer_flag[i]);
  }
  da.epoch = static_cast<uint32_t*>(d->epoch);
  da.done_counter = static_cast<unsigned int*>(d->done_counter);
  da.status = static_cast<int*>(d->status);
  da.trace = static_cast<unsigned long long*>(d->trace);
  // tensor-core GEMV: bf16 gate, expert tiles that divide the 32 warps, H slices of whole 128-column steps
  const int et = (r->E + 15) / 16;
  const int nsplit = et <= 32 ? 32 / et : 0;
  a.mma_logits = (!r->gate_fp32 && nsplit >= 1 && (et & (et - 1)) == 0 && d->H % (128 * nsplit) == 0) ? 1 : 0;
  const size_t smem = static_cast<size_t>(d->H) * 2 + (r->E + 32) * sizeof(float) +
                      (a.mma_logits ? static_cast<size_t>(nsplit) * et * 16 * sizeof(float) : 0);
  ag_route_dispatch_kernel<<<d->T, 1024, smem, static_cast<cudaStream_t>(stream)>>>(a);
  AFD_CHECK_LAUNCH();
  return 0;
}

struct AfdGroupDesc {
  const void* recv_idx; const void* n2m_flag; void* epoch;
  int A, T, K, recv_tokens, expert_base, experts_local, block_tok, pool_rows, max_tok_tiles;
  void* row_meta; void* tile_info; void* counters; void* expert_counts;
  unsigned long long timeout_ns;
  void* status;
  // gather
  const void* recv_x; const void* recv_scale; void* pool_x; void* pool_scale;
  int row_bytes, scale_per_row;
  void* trace;
  void* done_counter;   // device word (0) for the fused one-launch path; null = two-launch path
};

extern "C" int afd_eg_group_gather(const AfdGroupDesc* d, void* stream) {
  if (d->A > kMaxRanks || d->A > 1024 || d->T > 65535 || d->K > 255) return -1;
  if (d->row_bytes % 16 != 0) return -2;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GroupArgs g{};
  g.recv_idx = static_cast<const int*>(d->recv_idx);
  g.n2m_flag = static_cast<const uint32_t*>(d->n2m_flag);
  g.epoch = static_cast<uint32_t*>(d->epoch);
  g.A = d->A; g.T = d->T; g.K = d->K; g.recv_tokens = d->recv_tokens;
  g.expert_base = d->expert_base; g.experts_local = d->experts_local; g.block_tok = d->block_tok;
  g.pool_rows = d->pool_rows; g.max_tok_tiles = d->max_tok_tiles;
  g.row_meta = static_cast<uint32_t*>(d->row_meta);
  g.tile_info = static_cast<int4*>(d->tile_info);
  g.counters = static_cast<int*>(d->counters);
  g.expert_counts = static_cast<int*>(d->expert_counts);
  g.timeout_ns = d->timeout_ns;
  g.status = static_cast<int*>(d->status);
  g.trace = static_cast<unsigned long long*>(d->trace);
  if (static_cast<long>(d->A) * d->T * d->K <= kFusedGroupMaxEntries && d->block_tok <= 128 && d->done_counter != nullptr) {
    FusedGroupArgs fa{};
    fa.g = g;
    fa.recv_x = d->recv_x; fa.recv_scale = static_cast<const float*>(d->recv_scale);
    fa.pool_x = d->pool_x; fa.pool_scale = static_cast<float*>(d->pool_scale);
    fa.row_bytes = d->row_bytes; fa.scale_per_row = d->scale_per_row;
    fa.done_counter = static_cast<unsigned int*>(d->done_counter);
    // every possible tile gets a CTA: at most ceil(entries / block_tok) + experts_local tiles
    const long entries = static_cast<long>(d->A) * d->T * d->K;
    int grid = static_cast<int>((entries + d->block_tok - 1) / d->block_tok) + d->experts_local;
    if (grid > d->max_tok_tiles) grid = d->max_tok_tiles;
    eg_group_gather_fused_kernel<<<grid, kFusedGroupThreads, (2 * d->experts_local + 1) * sizeof(int), st>>>(fa);
    AFD_CHECK_LAUNCH();
    return 0;
  }
  eg_group_kernel<<<1, 1024, 3 * d->experts_local * sizeof(int), st>>>(g);
  AFD_CHECK_LAUNCH();
  GatherArgs ga{};
  ga.recv_x = d->recv_x; ga.recv_scale = static_cast<const float*>(d->recv_scale);
  ga.row_meta = g.row_meta; ga.tile_info = g.tile_info; ga.counters = g.counters;
  ga.pool_x = d->pool_x; ga.pool_scale = static_cast<float*>(d->pool_scale);
  ga.recv_tokens = d->recv_tokens; ga.row_bytes = d->row_bytes; ga.scale_per_row = d->scale_per_row;
  ga.block_tok = d->block_tok; ga.max_tok_tiles = d->max_tok_tiles;
  const int grid = d->max_tok_tiles < 592 ? d->max_tok_tiles : 592;
  eg_gather_kernel<<<grid, 256, 0, st>>>(ga);
  AFD_CHECK_LAUNCH();
  return 0;
}

struct AfdCombineDesc {
  const void* combine; const void* topk_w; const void* topk_idx; const void* m2n_flag;
  void* epoch; void* done_counter;
  int T, H, K, combine_tokens, num_eg;
  float scale;
  const void* extra; void* y; void* residual; const void* norm_w; void* normed;
  float eps; int offset1;
  unsigned long long timeout_ns;
  void* status;
  void* trace;
};

extern "C" int afd_ag_combine(const AfdCombineDesc* d, void* stream) {
  if (d->T == 0) return -1;
  if (d->H % 8 != 0 || d->num_eg > kMaxRanks) return -2;
  CombineArgs a{};
  a.combine = static_cast<const __nv_bfloat16*>(d->combine);
  a.topk_w = static_cast<const float*>(d->topk_w);
  a.topk_idx = static_cast<const int*>(d->topk_idx);
  a.m2n_flag = static_cast<const uint32_t*>(d->m2n_flag);
  a.epoch = static_cast<uint32_t*>(d->epoch);
  a.done_counter = static_cast<unsigned int*>(d->done_counter);
  a.T = d->T; a.H = d->H; a.K = d->K; a.combine_tokens = d->combine_tokens; a.num_eg = d->num_eg;
  a.scale = d->scale;
  a.extra = static_cast<const __nv_bfloat16*>(d->extra);
  a.y = static_cast<__nv_bfloat16*>(d->y);
  a.residual = static_cast<__nv_bfloat16*>(d->residual);
  a.norm_w = static_cast<const __nv_bfloat16*>(d->norm_w);
  a.normed = static_cast<__nv_bfloat16*>(d->normed);
  a.eps = d->eps; a.offset1 = d->offset1; a.timeout_ns = d->timeout_ns;
  a.status = static_cast<int*>(d->status);
  a.trace = static_cast<unsigned long long*>(d->trace);
  const int threads = d->H / 8 >= 512 ? 512 : 256;
  cudaError_t le = launch_pdl(ag_combine_kernel, dim3(d->T), dim3(threads), (d->H + 32) * sizeof(float),
                              static_cast<cudaStream_t>(stream), 1, a);
  if (le != cudaSuccess) return static_cast<int>(le);
  return 0;
}

extern "C" int afd_wait_flag(const void* flag, unsigned int target, unsigned long long timeout_ns,
                             void* status, void* stream) {
  wait_flag_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint32_t*>(flag), target, timeout_ns, static_cast<int*>(status));
  AFD_CHECK_LAUNCH();
  return 0;
}

extern "C" int afd_set_flag(void* flag, unsigned int value, void* stream) {
  set_flag_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint32_t*>(flag), value);
  AFD_CHECK_LAUNCH();
  return 0;
}
