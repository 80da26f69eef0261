// Router building blocks shared by the fused route + dispatch kernels: the m16n8k16 tensor-core
// step used for the router logits, the warp-wide scoring + top-k selection, and the 1x128 FP8
// quantisation of one row group.
#pragma once

#include "common.cuh"

namespace afd {

__device__ __forceinline__ void mma_gemv_16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}


template <int MAX_PER_LANE>
__device__ __forceinline__ void warp_topk(const float* s_logit, const float* bias, int E, int K, int scoring,
                                          int renorm, float scale, int* out_idx, float* out_w, int lane) {
  float sc[MAX_PER_LANE], sel[MAX_PER_LANE];
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < MAX_PER_LANE; ++j) {
    const int e = j * 32 + lane;
    sc[j] = e < E ? s_logit[e] : -INFINITY;
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
  float wsum = 0.f, my_w = 0.f;
  int my_i = 0;
  for (int k = 0; k < K; ++k) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < MAX_PER_LANE; ++j) {
      if (sel[j] > best) {
        best = sel[j];
        bi = j * 32 + lane;
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
    wv = warp_sum(wv);
    wsum += wv;
    if (lane == k) {
      my_w = wv;
      my_i = bi;
    }
  }
  const float mul = (renorm ? 1.f / fmaxf(wsum, 1e-20f) : 1.f) * scale;
  if (lane < K) {
    out_idx[lane] = my_i;
    out_w[lane] = my_w * mul;
  }
}

// ---- thread-block cluster helpers (a kernel launched without a cluster is a cluster of one) ----
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

}  // namespace afd
