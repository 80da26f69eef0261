// Decode-sized N2M exchange that lands where the expert GEMM reads it.
//
// The expert GPU keeps, per lane, a pool with a fixed stripe of `cap` rows for every local
// expert, one slot counter per expert, and a row_meta word per pool row. An attention rank
// routes a token, claims one slot per chosen expert with a (remote) atomic add on that expert's
// counter and stores the row, its meta word and (FP8) its 1x128 scales straight into the slot.
// The last CTA releases the rank's flag on every expert GPU, as in the receive-slot protocol.
// The expert GPU then only has to turn the counters into a tile schedule: no grouping pass over
// the received ids and no gather copy through HBM. Slot order inside an expert depends on the
// order of the atomics; results do not, because every pool row is computed independently and
// carries its own (source, k, token) destination.
//
//   ag_route_direct_kernel  post-attention step of an attention rank for TPC tokens per CTA:
//       residual += attn_out; x = RMSNorm(residual); router logits on tensor cores with the TPC
//       tokens as the MMA N side (the gate matrix is read once per TPC tokens, and the expert
//       range can be split over a thread-block cluster whose CTAs send their logits to CTA 0
//       through distributed shared memory); scoring + top-k; slot claim; row push; flag release.
//   dispatch_direct_kernel  the same push for a routing that was computed elsewhere.
//   eg_schedule_kernel      expert side: bounded wait for the sources' flags, counters -> tile
//       schedule for the grouped GEMMs, counters back to zero for the lane's next round.
//
// Reference behaviour: tokens landing in expert-grouped pool blocks and arrival counts driving
// the GEMM, python/minisgl/kernel/csrc/deepgemm/deep_gemm/include/deep_gemm/impls/sm100_mega_moe_m2n.cuh:2023-2254,2363-2441;
// the fused tensor-core router python/minisgl/kernel/csrc/jit/gate_topk_fused.cu.
#include "common.cuh"
#include "route_common.cuh"

namespace afd {

constexpr int kMaxDirectRanks = 16;
constexpr int kRouteThreads = 512;
constexpr int kMaxTopk = 32;

struct DirectArgs {
  void* peer_pool[kMaxDirectRanks];          // [E_local * cap][row_bytes] on each expert GPU
  float* peer_scale[kMaxDirectRanks];        // fp8: [E_local * cap][H / 128]
  uint32_t* peer_meta[kMaxDirectRanks];      // [E_local * cap]: src << 24 | k << 16 | token
  uint32_t* peer_count[kMaxDirectRanks];     // [E_local] slot counters
  uint32_t* peer_flag[kMaxDirectRanks];      // this source's flag word on each expert GPU
  int num_eg, experts_per_eg, cap, fp8;
  int T, H, K, src_rank;
  uint32_t* epoch;
  unsigned int* done_counter;
  int* status;
  unsigned long long* trace;
};

__device__ __forceinline__ unsigned int atomic_add_sys(uint32_t* p, unsigned int v) {
  unsigned int old;
  asm volatile("atom.relaxed.sys.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Claim a slot for (token t, choice k, expert e): returns the destination as eg << 24 | pool row,
// or 0xffffffff when the expert id is out of range or its stripe is full (status is set).
__device__ __forceinline__ uint32_t claim_slot(const DirectArgs& d, int t, int k, int e) {
  if (e < 0) return 0xffffffffu;
  const int eg = e / d.experts_per_eg, el = e - eg * d.experts_per_eg;
  if (eg >= d.num_eg) {
    set_status(d.status, kStatusBadExtent);
    return 0xffffffffu;
  }
  const unsigned int slot = atomic_add_sys(d.peer_count[eg] + el, 1u);
  if (slot >= static_cast<unsigned int>(d.cap)) {
    set_status(d.status, kStatusCapacity);
    return 0xffffffffu;
  }
  const uint32_t row = static_cast<uint32_t>(el) * d.cap + slot;
  d.peer_meta[eg][row] = (static_cast<uint32_t>(d.src_rank) << 24) | (static_cast<uint32_t>(k) << 16) |
                         static_cast<uint32_t>(t);
  return (static_cast<uint32_t>(eg) << 24) | row;
}

// The last pushing CTA publishes this source's epoch on every expert GPU (data -> fence.gpu ->
// counter -> fence.sys -> flags), then advances the epoch. Returns whether this CTA was the last.
__device__ __forceinline__ bool release_flags(const DirectArgs& d, unsigned int pushing_ctas, bool local_only = false) {
  __threadfence();
  const unsigned int prev = atomicAdd(d.done_counter, 1u);
  const bool last = prev == pushing_ctas - 1;
  if (last) {
    // every consumer on this GPU (and ordered behind this kernel): a device-scope fence is enough
    if (local_only) __threadfence();
    else __threadfence_system();
    const uint32_t e = *d.epoch;
    for (int g = 0; g < d.num_eg; ++g) st_relaxed_sys(d.peer_flag[g], e);
    trace_stamp(d.trace, e, 0);
    *d.epoch = e + 1;
    *d.done_counter = 0;
    __threadfence();
  }
  return last;
}

// ---------------------------------------------------------------------------------------------
// Push with a given routing: one CTA per token.
// ---------------------------------------------------------------------------------------------
struct DispatchDirectArgs {
  const __nv_bfloat16* x;     // [T][H]
  const int* topk_idx;        // [T][K] global expert ids (< 0: no expert)
  DirectArgs d;
};

__global__ void __launch_bounds__(256) dispatch_direct_kernel(const DispatchDirectArgs a) {
  const DirectArgs& d = a.d;
  const int t = blockIdx.x, H = d.H;
  __shared__ uint32_t s_dst[kMaxTopk];
  extern __shared__ __align__(16) uint8_t dsm_raw[];     // fp8: quantised row + scales
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x < d.K) s_dst[threadIdx.x] = claim_slot(d, t, threadIdx.x, a.topk_idx[static_cast<size_t>(t) * d.K + threadIdx.x]);
  const __nv_bfloat16* xr = a.x + static_cast<size_t>(t) * H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (d.fp8) {
    uint8_t* xq = dsm_raw;
    float* xsc = reinterpret_cast<float*>(dsm_raw + H);
    for (int g = warp; g < H / 128; g += nw) {
      const uint2 raw = *reinterpret_cast<const uint2*>(xr + g * 128 + lane * 4);
      const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
      const float2 f0 = __bfloat1622float2(b2[0]), f1 = __bfloat1622float2(b2[1]);
      float amax = fmaxf(fmaxf(fabsf(f0.x), fabsf(f0.y)), fmaxf(fabsf(f1.x), fabsf(f1.y)));
      amax = warp_max(amax);
      const float scale = fmaxf(amax, 1e-10f) / 448.f, inv = 1.f / scale;
      uint32_t packed = 0;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f0.x * inv, __NV_SATFINITE, __NV_E4M3));
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f0.y * inv, __NV_SATFINITE, __NV_E4M3)) << 8;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f1.x * inv, __NV_SATFINITE, __NV_E4M3)) << 16;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(f1.y * inv, __NV_SATFINITE, __NV_E4M3)) << 24;
      *reinterpret_cast<uint32_t*>(xq + g * 128 + lane * 4) = packed;
      if (lane == 0) xsc[g] = scale;
    }
  }
  __syncthreads();
  const int row_bytes = d.fp8 ? H : H * 2;
  const int vec = row_bytes / 16;
  const uint8_t* src = d.fp8 ? dsm_raw : reinterpret_cast<const uint8_t*>(xr);
  for (int idx = threadIdx.x; idx < d.K * vec; idx += blockDim.x) {
    const int k = idx / vec, v = idx - k * vec;
    const uint32_t dst = s_dst[k];
    if (dst == 0xffffffffu) continue;
    const uint4 val = *reinterpret_cast<const uint4*>(src + v * 16);
    uint8_t* base = static_cast<uint8_t*>(d.peer_pool[dst >> 24]) + static_cast<size_t>(dst & 0xffffffu) * row_bytes;
    reinterpret_cast<uint4*>(base)[v] = val;
  }
  if (d.fp8) {
    const float* xsc = reinterpret_cast<const float*>(dsm_raw + H);
    const int groups = H / 128;
    for (int idx = threadIdx.x; idx < d.K * groups; idx += blockDim.x) {
      const int k = idx / groups, g = idx - k * groups;
      const uint32_t dst = s_dst[k];
      if (dst == 0xffffffffu) continue;
      d.peer_scale[dst >> 24][static_cast<size_t>(dst & 0xffffffu) * groups + g] = xsc[g];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) release_flags(d, gridDim.x);
}

// ---------------------------------------------------------------------------------------------
// Expert side: flags -> tile schedule. One warp.
// ---------------------------------------------------------------------------------------------
struct ScheduleArgs {
  const uint32_t* n2m_flag;   // [A]
  int A;
  uint32_t* epoch;            // expected epoch; advanced here
  uint32_t* counts;           // [experts_local] slot counters, reset here
  int experts_local, cap, block_tok, max_tok_tiles;
  int4* tile_info;            // {expert, first pool row, valid rows, 0}
  int* counters;              // [0] tiles, [1] padded rows, [2] routed rows
  int* expert_counts;         // optional copy of the counts (load statistics)
  uint64_t timeout_ns;
  int* status;
  unsigned long long* trace;
};

// One warp turns the slot counters into the tile schedule and clears them. `wait`: first wait
// (bounded) for every source's flag; without it the caller guarantees that all sources are done
// (the single source's own last CTA, when attention and experts share the GPU).
__device__ __forceinline__ void schedule_warp(const ScheduleArgs& a, int lane, bool wait) {
  const uint32_t e0 = *a.epoch;
  if (lane == 0) trace_stamp(a.trace, e0, 0);
  if (wait && lane < a.A) wait_flag_ge(a.n2m_flag + lane, e0, a.timeout_ns, a.status);
  __syncwarp();
  __threadfence();
  if (lane == 0) trace_stamp(a.trace, e0, 1);
  const int per = (a.experts_local + 31) / 32;
  const int lo = min(lane * per, a.experts_local), hi = min(lo + per, a.experts_local);
  constexpr int kMaxPer = 16;             // 512 local experts at most (host check)
  int cs[kMaxPer];
  int tiles = 0, routed = 0;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lo + i;
    int c = (i < per && e < hi) ? static_cast<int>(__ldcg(a.counts + e)) : 0;
    if (c > a.cap) c = a.cap;             // a source that overran the stripe has set the status
    cs[i] = c;
    tiles += (c + a.block_tok - 1) / a.block_tok;
    routed += c;
  }
  int incl = tiles, rincl = routed;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    const int vr = __shfl_up_sync(0xffffffffu, rincl, o);
    if (lane >= o) {
      incl += v;
      rincl += vr;
    }
  }
  int t = incl - tiles;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    const int e = lo + i;
    if (i < per && e < hi) {
      const int c = cs[i];
      if (a.expert_counts) a.expert_counts[e] = c;
      a.counts[e] = 0;                    // the lane's next round starts from empty stripes
      for (int j = 0; j * a.block_tok < c; ++j, ++t) {
        if (t < a.max_tok_tiles) a.tile_info[t] = make_int4(e, e * a.cap + j * a.block_tok, min(a.block_tok, c - j * a.block_tok), 0);
      }
    }
  }
  if (lane == 31) {
    int total = incl;
    if (total > a.max_tok_tiles) {
      set_status(a.status, kStatusCapacity);
      total = a.max_tok_tiles;
    }
    a.counters[0] = total;
    a.counters[1] = total * a.block_tok;
    a.counters[2] = rincl;
    trace_stamp(a.trace, e0, 2);
    *a.epoch = e0 + 1;
  }
}

__global__ void __launch_bounds__(32) eg_schedule_kernel(const ScheduleArgs a) {
  pdl_trigger();
  pdl_wait();
  schedule_warp(a, threadIdx.x, true);
}

// ---------------------------------------------------------------------------------------------
// Fused post-attention step with direct dispatch.
// ---------------------------------------------------------------------------------------------
struct RouteDirectArgs {
  const __nv_bfloat16* attn_out;   // [T][H]
  __nv_bfloat16* residual;         // [T][H] in/out
  const __nv_bfloat16* norm_w;     // [H]
  const void* gate_w;              // [E][H] bf16 or fp32
  const float* gate_bias;          // [E] or null
  __nv_bfloat16* x_out;            // [T][H] normed hidden (local copy for the shared expert)
  int* topk_idx_out;               // [T][K]
  float* topk_w_out;               // [T][K]
  int E, gate_fp32, scoring, renorm, offset1, mma_logits;
  float eps, route_scale;
  DirectArgs d;
  // Attention and experts on one GPU, a single source: the last pushing CTA also builds the expert
  // side's tile schedule (one launch less in front of the grouped GEMMs).
  int fuse_schedule;
  ScheduleArgs sched;
};

// Dynamic shared memory, in order:
//   xs      [TPC][H + 32] bf16   normed rows (64 bytes of padding per row: conflict-free B loads)
//   s_logit [TPC][E] fp32        complete logits (CTA 0 of the cluster receives every slice)
//   s_part  [nsplit][TPC][E_cta] fp32   partial logits of the K slices (tensor-core path)
//   s_ss    [TPC * H / 256] fp32 per-warp sums of squares
//   s_xq    fp8: [TPC][H] bytes + [TPC][H/128] fp32 scales (CTA 0)
template <int TPC>
__global__ void __launch_bounds__(kRouteThreads) ag_route_direct_kernel(const RouteDirectArgs a) {
  extern __shared__ __align__(16) uint8_t rsm[];
  const DirectArgs& d = a.d;
  const int H = d.H, E = a.E, K = d.K;
  const int XS = H + 32;
  const uint32_t crank = cluster_ctarank(), csize = cluster_nctarank();
  const int group = blockIdx.x / csize;                 // token group of this cluster
  const int ngroups = gridDim.x / csize;
  const int tok0 = group * TPC;
  const int ntok = min(TPC, d.T - tok0);                // valid tokens of this group
  const int e_cta = E / static_cast<int>(csize);        // experts scored by this CTA
  const int e_lo = static_cast<int>(crank) * e_cta;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NW = kRouteThreads / 32;

  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(rsm);
  float* s_logit = reinterpret_cast<float*>(rsm + static_cast<size_t>(TPC) * XS * 2);
  float* s_part = s_logit + TPC * E;
  const int ET = (e_cta + 15) >> 4;
  const int nsplit = a.mma_logits ? max(1, NW / ET) : 0;
  float* s_ss = s_part + nsplit * TPC * ET * 16;
  uint8_t* s_xq = reinterpret_cast<uint8_t*>(s_ss + TPC * (H / 256));
  __shared__ int s_idx[TPC][kMaxTopk];
  __shared__ float s_w[TPC][kMaxTopk];
  __shared__ uint32_t s_dst[TPC][kMaxTopk];

  // 0. pull this CTA's gate slice towards L2 (weights: independent of the predecessor kernel)
  pdl_trigger();
  {
    const size_t row_b = static_cast<size_t>(H) * (a.gate_fp32 ? 4 : 2);
    const char* gp = static_cast<const char*>(a.gate_w) + static_cast<size_t>(e_lo) * row_b;
    const size_t bytes = static_cast<size_t>(e_cta) * row_b;
    const size_t per = (bytes / ngroups + 127) / 128 * 128;
    const size_t lo = per * group, hi = min(bytes, lo + per);
    for (size_t off = lo + static_cast<size_t>(tid) * 128; off < hi; off += static_cast<size_t>(kRouteThreads) * 128) {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(gp + off));
    }
  }

  pdl_wait();
  // 1. residual add + RMSNorm of the group's rows. Every CTA of the cluster computes the rows (it
  //    needs them for its logits); CTA 0 alone writes residual and x_out, and only after all CTAs
  //    have loaded the old residual (cluster barrier between the loads and the stores).
  const int vec_per_row = H / 8;                        // uint4 per row; a multiple of 32 (H % 256 == 0)
  const int nvec = ntok * vec_per_row;
  constexpr int MAXV = (TPC * 4096 / 8 + kRouteThreads - 1) / kRouteThreads;    // H <= 4096
  uint4 rnew[MAXV];
#pragma unroll
  for (int p = 0; p < MAXV; ++p) {
    const int idx = p * kRouteThreads + tid;
    float ss = 0.f;
    if (idx < nvec) {
      const int tk = idx / vec_per_row, c = idx - tk * vec_per_row;
      const size_t off = static_cast<size_t>(tok0 + tk) * H + c * 8;
      const uint4 xa = *reinterpret_cast<const uint4*>(a.attn_out + off);
      uint4 ra = *reinterpret_cast<const uint4*>(a.residual + off);
      const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xa);
      __nv_bfloat162* r2 = reinterpret_cast<__nv_bfloat162*>(&ra);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 xv = __bfloat1622float2(x2[j]);
        float2 rv = __bfloat1622float2(r2[j]);
        r2[j] = __floats2bfloat162_rn(rv.x + xv.x, rv.y + xv.y);
        rv = __bfloat1622float2(r2[j]);
        ss += rv.x * rv.x + rv.y * rv.y;
      }
      rnew[p] = ra;
    }
    ss = warp_sum(ss);
    if (lane == 0 && p * kRouteThreads + warp * 32 < nvec) s_ss[p * NW + warp] = ss;
  }
  cluster_arrive();            // this CTA's loads of the old residual are done
  __syncthreads();
  cluster_wait();
  const int warps_per_row = vec_per_row / 32;
#pragma unroll
  for (int p = 0; p < MAXV; ++p) {
    const int idx = p * kRouteThreads + tid;
    if (idx < nvec) {
      const int tk = idx / vec_per_row, c = idx - tk * vec_per_row;
      float tot = 0.f;
      for (int w = 0; w < warps_per_row; ++w) tot += s_ss[tk * warps_per_row + w];
      const float inv = rsqrtf(tot / H + a.eps);
      const size_t off = static_cast<size_t>(tok0 + tk) * H + c * 8;
      const uint4 wa = *reinterpret_cast<const uint4*>(a.norm_w + c * 8);
      const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&wa);
      const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rnew[p]);
      uint4 oa;
      __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&oa);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 g = __bfloat1622float2(w2[j]);
        if (a.offset1) {
          g.x += 1.f;
          g.y += 1.f;
        }
        const float2 rv = __bfloat1622float2(r2[j]);
        o2[j] = __floats2bfloat162_rn(rv.x * inv * g.x, rv.y * inv * g.y);
      }
      *reinterpret_cast<uint4*>(xs + tk * XS + c * 8) = oa;      // the router sees the bf16-rounded x
      if (crank == 0) {
        *reinterpret_cast<uint4*>(a.residual + off) = rnew[p];
        *reinterpret_cast<uint4*>(a.x_out + off) = oa;
      }
    }
  }
  // rows of missing tokens (last group) read as zeros
  for (int idx = nvec + tid; idx < TPC * vec_per_row; idx += kRouteThreads) {
    const int tk = idx / vec_per_row, c = idx - tk * vec_per_row;
    *reinterpret_cast<uint4*>(xs + tk * XS + c * 8) = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();

  // 2. logits of experts [e_lo, e_lo + e_cta) for the TPC tokens
  const uint32_t logit0 = cluster_map(smem_u32(s_logit), 0);     // CTA 0's logits (this CTA's when alone)
  if (a.mma_logits) {
    // A warp owns 16 experts (MMA M) over one K slice; the tokens are the MMA N side. A lane loads
    // 16 contiguous bytes of two gate rows per 32 columns and the same columns of its token's row,
    // so the columns meet in a permuted order that is the same for both operands.
    const int g = lane >> 2, t4 = lane & 3;
    const int tokrow = (TPC == 8 ? g : (g & (TPC - 1))) * XS;
    for (int job = warp; job < ET * nsplit; job += NW) {
      int et = job % ET + (group % ET);                  // groups start at different expert tiles
      if (et >= ET) et -= ET;
      const int ks = job / ET;
      const int kb0 = ks * (H / 32 / nsplit), kb1 = kb0 + H / 32 / nsplit;
      const int r_lo = e_lo + min(et * 16 + g, e_cta - 1), r_hi = e_lo + min(et * 16 + g + 8, e_cta - 1);
      const __nv_bfloat16* g_lo = static_cast<const __nv_bfloat16*>(a.gate_w) + static_cast<size_t>(r_lo) * H + t4 * 8;
      const __nv_bfloat16* g_hi = static_cast<const __nv_bfloat16*>(a.gate_w) + static_cast<size_t>(r_hi) * H + t4 * 8;
      float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
      for (int kb = kb0; kb < kb1; kb += 4) {            // slices are whole groups of 4 (host check)
        uint4 lo[4], hi[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          lo[u] = __ldg(reinterpret_cast<const uint4*>(g_lo + (kb + u) * 32));
          hi[u] = __ldg(reinterpret_cast<const uint4*>(g_hi + (kb + u) * 32));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const uint4 xv = *reinterpret_cast<const uint4*>(xs + tokrow + (kb + u) * 32 + t4 * 8);
          mma_gemv_16816(c, lo[u].x, hi[u].x, lo[u].y, hi[u].y, xv.x, xv.y);
          mma_gemv_16816(c, lo[u].z, hi[u].z, lo[u].w, hi[u].w, xv.z, xv.w);
        }
      }
      // c0/c1: expert row g, tokens 2*t4, 2*t4+1; c2/c3: expert row g + 8
      float* part = s_part + static_cast<size_t>(ks) * TPC * ET * 16;
      const int tk = t4 * 2;
      if (tk < TPC) {
        part[tk * ET * 16 + et * 16 + g] = c[0];
        part[tk * ET * 16 + et * 16 + g + 8] = c[2];
      }
      if (tk + 1 < TPC) {
        part[(tk + 1) * ET * 16 + et * 16 + g] = c[1];
        part[(tk + 1) * ET * 16 + et * 16 + g + 8] = c[3];
      }
    }
    __syncthreads();
    for (int i = tid; i < TPC * e_cta; i += kRouteThreads) {
      const int tk = i / e_cta, e = i - tk * e_cta;
      float v = 0.f;
      for (int ks = 0; ks < nsplit; ++ks) v += s_part[(static_cast<size_t>(ks) * TPC + tk) * ET * 16 + e];
      st_cluster_f32(logit0 + static_cast<uint32_t>(tk * E + e_lo + e) * 4u, v);
    }
  } else {
    // One warp per expert row, lanes split H, every token's dot product from one read of the row.
    for (int e = warp; e < e_cta; e += NW) {
      float acc[TPC];
#pragma unroll
      for (int tk = 0; tk < TPC; ++tk) acc[tk] = 0.f;
      if (a.gate_fp32) {
        const float* gr = static_cast<const float*>(a.gate_w) + static_cast<size_t>(e_lo + e) * H;
#pragma unroll 2
        for (int i = lane * 8; i < H; i += 256) {
          const float4 g0 = __ldg(reinterpret_cast<const float4*>(gr + i));
          const float4 g1 = __ldg(reinterpret_cast<const float4*>(gr + i + 4));
#pragma unroll
          for (int tk = 0; tk < TPC; ++tk) {
            const uint4 xa = *reinterpret_cast<const uint4*>(xs + tk * XS + i);
            const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xa);
            const float2 a0 = __bfloat1622float2(x2[0]), a1 = __bfloat1622float2(x2[1]);
            const float2 a2 = __bfloat1622float2(x2[2]), a3 = __bfloat1622float2(x2[3]);
            acc[tk] += g0.x * a0.x + g0.y * a0.y + g0.z * a1.x + g0.w * a1.y + g1.x * a2.x + g1.y * a2.y + g1.z * a3.x + g1.w * a3.y;
          }
        }
      } else {
        const __nv_bfloat16* gr = static_cast<const __nv_bfloat16*>(a.gate_w) + static_cast<size_t>(e_lo + e) * H;
#pragma unroll 2
        for (int i = lane * 8; i < H; i += 256) {
          const uint4 ga = __ldg(reinterpret_cast<const uint4*>(gr + i));
          const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&ga);
#pragma unroll
          for (int tk = 0; tk < TPC; ++tk) {
            const uint4 xa = *reinterpret_cast<const uint4*>(xs + tk * XS + i);
            const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&xa);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 gv = __bfloat1622float2(g2[j]), xv = __bfloat1622float2(x2[j]);
              acc[tk] = fmaf(gv.x, xv.x, acc[tk]);
              acc[tk] = fmaf(gv.y, xv.y, acc[tk]);
            }
          }
        }
      }
#pragma unroll
      for (int tk = 0; tk < TPC; ++tk) {
        const float v = warp_sum(acc[tk]);
        if (lane == 0) st_cluster_f32(logit0 + static_cast<uint32_t>(tk * E + e_lo + e) * 4u, v);
      }
    }
  }
  cluster_arrive();            // this CTA's logits are in CTA 0's shared memory
  cluster_wait();
  if (crank != 0) return;

  // 3. scoring + top-k: warp w takes token w; then one thread per (token, choice) claims a slot
  if (warp < ntok) {
    const float* lg = s_logit + warp * E;
    if (E <= 128) warp_topk<4>(lg, a.gate_bias, E, K, a.scoring, a.renorm, a.route_scale, s_idx[warp], s_w[warp], lane);
    else if (E <= 256) warp_topk<8>(lg, a.gate_bias, E, K, a.scoring, a.renorm, a.route_scale, s_idx[warp], s_w[warp], lane);
    else warp_topk<16>(lg, a.gate_bias, E, K, a.scoring, a.renorm, a.route_scale, s_idx[warp], s_w[warp], lane);
    __syncwarp();
    if (lane < K) {
      const int t = tok0 + warp, e = s_idx[warp][lane];
      a.topk_idx_out[static_cast<size_t>(t) * K + lane] = e;
      a.topk_w_out[static_cast<size_t>(t) * K + lane] = s_w[warp][lane];
      s_dst[warp][lane] = claim_slot(d, t, lane, e);
    }
  }
  // FP8: quantise each row once (1x128 groups), all warps
  const int groups = H / 128;
  if (d.fp8) {
    float* s_sc = reinterpret_cast<float*>(s_xq + static_cast<size_t>(TPC) * H);
    for (int job = warp; job < ntok * groups; job += NW) {
      const int tk = job / groups, g128 = job - tk * groups;
      const uint2 fr = *reinterpret_cast<const uint2*>(xs + tk * XS + g128 * 128 + lane * 4);
      const __nv_bfloat162* f2 = reinterpret_cast<const __nv_bfloat162*>(&fr);
      const float2 fa = __bfloat1622float2(f2[0]), fb = __bfloat1622float2(f2[1]);
      float amax = fmaxf(fmaxf(fabsf(fa.x), fabsf(fa.y)), fmaxf(fabsf(fb.x), fabsf(fb.y)));
      amax = warp_max(amax);
      const float scale = fmaxf(amax, 1e-10f) / 448.f, is = 1.f / scale;
      uint32_t packed = 0;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(fa.x * is, __NV_SATFINITE, __NV_E4M3));
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(fa.y * is, __NV_SATFINITE, __NV_E4M3)) << 8;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(fb.x * is, __NV_SATFINITE, __NV_E4M3)) << 16;
      packed |= static_cast<uint32_t>(__nv_cvt_float_to_fp8(fb.y * is, __NV_SATFINITE, __NV_E4M3)) << 24;
      *reinterpret_cast<uint32_t*>(s_xq + tk * H + g128 * 128 + lane * 4) = packed;
      if (lane == 0) s_sc[tk * groups + g128] = scale;
    }
  }
  __syncthreads();

  // 4. push every row into its K slots
  const int row_bytes = d.fp8 ? H : H * 2;
  const int vec = row_bytes / 16;
  for (int idx = tid; idx < ntok * K * vec; idx += kRouteThreads) {
    const int v = idx % vec, tkk = idx / vec;
    const int tk = tkk / K, k = tkk - tk * K;
    const uint32_t dst = s_dst[tk][k];
    if (dst == 0xffffffffu) continue;
    const uint4 val = d.fp8 ? *reinterpret_cast<const uint4*>(s_xq + tk * H + v * 16)
                            : *reinterpret_cast<const uint4*>(xs + tk * XS + v * 8);
    uint8_t* base = static_cast<uint8_t*>(d.peer_pool[dst >> 24]) + static_cast<size_t>(dst & 0xffffffu) * row_bytes;
    reinterpret_cast<uint4*>(base)[v] = val;
  }
  if (d.fp8) {
    const float* s_sc = reinterpret_cast<const float*>(s_xq + static_cast<size_t>(TPC) * H);
    for (int idx = tid; idx < ntok * K * groups; idx += kRouteThreads) {
      const int g = idx % groups, tkk = idx / groups;
      const int tk = tkk / K, k = tkk - tk * K;
      const uint32_t dst = s_dst[tk][k];
      if (dst == 0xffffffffu) continue;
      d.peer_scale[dst >> 24][static_cast<size_t>(dst & 0xffffffu) * groups + g] = s_sc[tk * groups + g];
    }
  }
  __syncthreads();
  __shared__ int s_last;
  if (tid == 0) s_last = release_flags(d, static_cast<unsigned int>(ngroups), a.fuse_schedule != 0) ? 1 : 0;
  if (a.fuse_schedule) {
    __syncthreads();
    if (s_last && warp == 0) schedule_warp(a.sched, lane, false);
  }
}

}  // namespace afd

using namespace afd;

struct AfdDirectDesc {
  void* peer_pool[kMaxDirectRanks]; void* peer_scale[kMaxDirectRanks]; void* peer_meta[kMaxDirectRanks];
  void* peer_count[kMaxDirectRanks]; void* peer_flag[kMaxDirectRanks];
  int num_eg, experts_per_eg, cap, fp8, T, H, K, src_rank;
  void* epoch; void* done_counter; void* status; void* trace;
};

static int fill_direct(DirectArgs& o, const AfdDirectDesc* d) {
  if (d->num_eg < 1 || d->num_eg > kMaxDirectRanks || d->K < 1 || d->K > kMaxTopk || d->H % 128 != 0 || d->T < 1 ||
      d->T > 65535 || d->cap < 1 || static_cast<long>(d->cap) * d->experts_per_eg > 0xffffffL)
    return -2;
  for (int i = 0; i < d->num_eg; ++i) {
    o.peer_pool[i] = d->peer_pool[i];
    o.peer_scale[i] = static_cast<float*>(d->peer_scale[i]);
    o.peer_meta[i] = static_cast<uint32_t*>(d->peer_meta[i]);
    o.peer_count[i] = static_cast<uint32_t*>(d->peer_count[i]);
    o.peer_flag[i] = static_cast<uint32_t*>(d->peer_flag[i]);
  }
  o.num_eg = d->num_eg; o.experts_per_eg = d->experts_per_eg; o.cap = d->cap; o.fp8 = d->fp8;
  o.T = d->T; o.H = d->H; o.K = d->K; o.src_rank = d->src_rank;
  o.epoch = static_cast<uint32_t*>(d->epoch);
  o.done_counter = static_cast<unsigned int*>(d->done_counter);
  o.status = static_cast<int*>(d->status);
  o.trace = static_cast<unsigned long long*>(d->trace);
  return 0;
}

extern "C" int afd_dispatch_direct(const void* x, const void* topk_idx, const AfdDirectDesc* d, void* stream) {
  DispatchDirectArgs a{};
  const int r = fill_direct(a.d, d);
  if (r != 0) return r;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.topk_idx = static_cast<const int*>(topk_idx);
  const size_t smem = d->fp8 ? static_cast<size_t>(d->H) + (d->H / 128) * sizeof(float) : 0;
  cudaError_t le = launch_pdl(dispatch_direct_kernel, dim3(d->T), dim3(256), smem, static_cast<cudaStream_t>(stream), 1, a);
  if (le != cudaSuccess) return static_cast<int>(le);
  return 0;
}

struct AfdRouteDirectDesc {
  const void* attn_out; void* residual; const void* norm_w; const void* gate_w; const void* gate_bias;
  void* x_out; void* topk_idx_out; void* topk_w_out;
  int E, gate_fp32, scoring, renorm, offset1;
  float eps, route_scale;
  int tokens_per_cta;      // 0 = choose; 4 or 8
  int cluster;             // 0 = choose; CTAs that share a token group's expert range (1, 2, 4, 8)
  AfdDirectDesc d;
  int fuse_schedule;       // 1: `sched` describes the expert side of the same GPU (single source)
  struct AfdScheduleDesc {
    const void* n2m_flag; int A; void* epoch; void* counts;
    int experts_local, cap, block_tok, max_tok_tiles;
    void* tile_info; void* counters; void* expert_counts;
    unsigned long long timeout_ns;
    void* status; void* trace;
  } sched;
};

static void fill_schedule(ScheduleArgs& a, const AfdRouteDirectDesc::AfdScheduleDesc* d) {
  a.n2m_flag = static_cast<const uint32_t*>(d->n2m_flag);
  a.A = d->A;
  a.epoch = static_cast<uint32_t*>(d->epoch);
  a.counts = static_cast<uint32_t*>(d->counts);
  a.experts_local = d->experts_local; a.cap = d->cap; a.block_tok = d->block_tok; a.max_tok_tiles = d->max_tok_tiles;
  a.tile_info = static_cast<int4*>(d->tile_info);
  a.counters = static_cast<int*>(d->counters);
  a.expert_counts = static_cast<int*>(d->expert_counts);
  a.timeout_ns = d->timeout_ns;
  a.status = static_cast<int*>(d->status);
  a.trace = static_cast<unsigned long long*>(d->trace);
}

template <int TPC>
static int launch_route_direct(const RouteDirectArgs& a, int cluster, size_t smem, cudaStream_t st) {
  auto kern = ag_route_direct_kernel<TPC>;
  static size_t smem_set = 0;
  if (smem > smem_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return static_cast<int>(e);
    smem_set = smem;
  }
  const int groups = (a.d.T + TPC - 1) / TPC;
  cudaError_t e = launch_pdl(kern, dim3(groups * cluster), dim3(kRouteThreads), smem, st, static_cast<unsigned int>(cluster), a);
  if (e != cudaSuccess) return static_cast<int>(e);
  return 0;
}

extern "C" int afd_ag_route_direct(const AfdRouteDirectDesc* r, void* stream) {
  RouteDirectArgs a{};
  const int rc = fill_direct(a.d, &r->d);
  if (rc != 0) return rc;
  const int H = r->d.H, E = r->E;
  if (H % 256 != 0 || H > 4096 || E < 1 || E > 512) return -2;
  a.attn_out = static_cast<const __nv_bfloat16*>(r->attn_out);
  a.residual = static_cast<__nv_bfloat16*>(r->residual);
  a.norm_w = static_cast<const __nv_bfloat16*>(r->norm_w);
  a.gate_w = r->gate_w;
  a.gate_bias = static_cast<const float*>(r->gate_bias);
  a.x_out = static_cast<__nv_bfloat16*>(r->x_out);
  a.topk_idx_out = static_cast<int*>(r->topk_idx_out);
  a.topk_w_out = static_cast<float*>(r->topk_w_out);
  a.E = E; a.gate_fp32 = r->gate_fp32; a.scoring = r->scoring; a.renorm = r->renorm; a.offset1 = r->offset1;
  a.eps = r->eps; a.route_scale = r->route_scale;
  a.fuse_schedule = 0;
  if (r->fuse_schedule) {
    if (r->d.num_eg != 1 || r->sched.A != 1 || r->sched.cap % r->sched.block_tok != 0 || r->sched.experts_local < 1 ||
        r->sched.experts_local > 512)
      return -5;
    a.fuse_schedule = 1;
    fill_schedule(a.sched, &r->sched);
  }
  // Measured on B200 (64 tokens, 128 experts, H 2048): 4 tokens per CTA with the expert range split
  // over 4 CTAs is the fastest form (more CTAs in flight, 128 KB of gate each).
  const int tpc = r->tokens_per_cta > 0 ? r->tokens_per_cta : 4;
  if (tpc != 4 && tpc != 8) return -3;
  int cluster = r->cluster;
  if (cluster <= 0) {
    const size_t gate_bytes = static_cast<size_t>(E) * H * (r->gate_fp32 ? 4 : 2);
    cluster = 1;
    while (cluster < 8 && gate_bytes / cluster > 128 * 1024 && E % (cluster * 2 * 16) == 0) cluster *= 2;
  }
  if (cluster != 1 && cluster != 2 && cluster != 4 && cluster != 8) return -4;
  if (E % cluster != 0) return -4;
  const int e_cta = E / cluster;
  const int nw = kRouteThreads / 32;
  const int et = (e_cta + 15) / 16;
  const int nsplit = et <= nw ? nw / et : 0;
  a.mma_logits = (!r->gate_fp32 && e_cta % 16 == 0 && nsplit >= 1 && (et & (et - 1)) == 0 && H % (128 * nsplit) == 0) ? 1 : 0;
  const int ns = a.mma_logits ? nsplit : 0;
  size_t smem = static_cast<size_t>(tpc) * (H + 32) * 2 + static_cast<size_t>(tpc) * E * 4 +
                static_cast<size_t>(ns) * tpc * et * 16 * 4 + static_cast<size_t>(tpc) * (H / 256) * 4;
  if (r->d.fp8) smem += static_cast<size_t>(tpc) * H + static_cast<size_t>(tpc) * (H / 128) * 4;
  smem = (smem + 15) / 16 * 16;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  return tpc == 8 ? launch_route_direct<8>(a, cluster, smem, st) : launch_route_direct<4>(a, cluster, smem, st);
}

typedef AfdRouteDirectDesc::AfdScheduleDesc AfdScheduleDesc;

extern "C" int afd_eg_schedule(const AfdScheduleDesc* d, void* stream) {
  if (d->A < 1 || d->A > 32 || d->cap % d->block_tok != 0 || d->experts_local < 1 || d->experts_local > 512) return -1;
  ScheduleArgs a{};
  fill_schedule(a, d);
  cudaError_t le = launch_pdl(eg_schedule_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), 1, a);
  if (le != cudaSuccess) return static_cast<int>(le);
  return 0;
}
