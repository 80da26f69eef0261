// Paged-KV grouped-query decode attention (flash-decoding with split KV), bf16 KV,
// head_dim 64 / 128 / 256, any page size, 1..N query tokens per request (N > 1 is the
// speculative-verify mode: query j of a request sees the first
// kv_len - q_len + 1 + j cached tokens).
//
// The op is bound by reading the KV cache once: every CTA owns one (request, kv head,
// 16-row query tile, KV split); each of its 4 warps streams its own 16-token
// KV tiles through a private 3-stage cp.async ring, computes S = Q K^T and O += P V
// with bf16 mma.sync (tensor throughput is not the limit here; bytes are) and keeps
// a private online-softmax state. Warps merge through shared memory; splits merge in
// the same launch: each split CTA writes its partial to an fp32 workspace and the last one
// to arrive (a counter per output tile, which it resets) combines them.
//
// Reference behaviour: the trtllm-gen paged decode call in
// python/minisgl/attention/trtllm.py:136-178 (bf16 KV, NHD pages, q_len_per_req for
// verify).
#include "common.cuh"

namespace afd {

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
constexpr int kMaxSplits = 32;   // bound of the split-merge weight table in shared memory

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

struct DecodeAttnArgs {
  const __nv_bfloat16* q;        // [B*q_len] rows of q_stride elements; heads [Hq][D] first
  long q_stride;
  const __nv_bfloat16* k_cache;  // [slots][Hkv][D]
  const __nv_bfloat16* v_cache;
  const int* page_table;         // [B][max_pages]
  const int* seq_lens;           // [B] KV length including the query tokens
  __nv_bfloat16* out;            // [B*q_len][Hq][D]
  float* part_o;                 // [B][Hkv][m_tiles][splits][16][D]
  float* part_lse;               // [B][Hkv][m_tiles][splits][16]
  unsigned int* part_count;      // [B][Hkv][m_tiles] arrival counters (zero between launches)
  int B, Hq, Hkv, q_len, page_size, page_shift, max_pages, splits, m_tiles;
  // Var-len mode (prefill chunks of several requests in one launch): request b owns the query rows
  // [q_starts[b], q_starts[b + 1]) of `q` / `out`; q_len is then the longest chunk (it sizes the grid).
  const int* q_starts;
  long cache_slots;
  float scale_log2;              // softmax scale * log2(e)
  int* status;
};

// Row-major [rows][D] bf16 tile in shared memory with 16-byte chunks XOR-swizzled by
// the row, so that ldmatrix reads are free of bank conflicts.
template <int D>
__device__ __forceinline__ uint32_t tile_off(int row, int chunk) {
  return static_cast<uint32_t>(row * D * 2 + ((chunk ^ (row & 7)) << 4));
}

template <int D>
struct AttnCfg {
  static constexpr int TOK = 16;                       // KV tokens per warp tile
  static constexpr int STAGES = 2;                     // cp.async ring depth per warp
  static constexpr int TILE_BYTES = TOK * D * 2;       // one of K / V
  static constexpr int WARP_BYTES = STAGES * 2 * TILE_BYTES;
  static constexpr int MERGE_BYTES = (16 * D + 32) * 4;
  static constexpr int WARP_REGION = WARP_BYTES > MERGE_BYTES ? WARP_BYTES : MERGE_BYTES;
  static constexpr int SMEM = 16 * D * 2 + 4 * WARP_REGION;
  static constexpr int CTAS_PER_SM = (222 * 1024) / (SMEM + 1024) >= 3 ? 3 : ((222 * 1024) / (SMEM + 1024) >= 2 ? 2 : 1);
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// NQ = query-row n-tiles per CTA (8 rows each): 1 when a (request, kv head) has at most 8
// query rows (decode with a GQA group of 8), else 2.
template <int D, int NQ>
__global__ void __launch_bounds__(128, AttnCfg<D>::CTAS_PER_SM) decode_attn_kernel(const DecodeAttnArgs a) {
  using Cfg = AttnCfg<D>;
  constexpr int ROWS = 8 * NQ;
  constexpr int TOK = Cfg::TOK;
  constexpr int CH = D / 8;            // 16-byte chunks per row
  constexpr int KT = D / 16;           // k-steps of S
  constexpr int TILE_BYTES = Cfg::TILE_BYTES;
  constexpr bool Q_REGS = D <= 128;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sq = smem;                          // Q tile 16 x D
  uint8_t* swarp = smem + 16 * D * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y / a.m_tiles, mt = blockIdx.y % a.m_tiles;
  const int b = blockIdx.z;
  const int G = a.Hq / a.Hkv;
  pdl_trigger();
  pdl_wait();
  int q_len = a.q_len;
  size_t q_base = static_cast<size_t>(b) * a.q_len;
  if (a.q_starts != nullptr) {
    q_base = static_cast<size_t>(a.q_starts[b]);
    q_len = a.q_starts[b + 1] - a.q_starts[b];
  }
  const int M = G * q_len;                     // valid query rows of this (b, kvh)
  if (mt * ROWS >= M) return;                  // var-len: a row tile past this request's rows (all its splits leave)
  int kv_len = a.seq_lens[b];
  if (kv_len < 0) kv_len = 0;
  if (kv_len > a.max_pages * a.page_size) {
    set_status(a.status, kStatusBadExtent);
    kv_len = a.max_pages * a.page_size;
  }

  // ---- stage Q (rows = j*G + g), zero for padding rows ----
  for (int idx = threadIdx.x; idx < 16 * CH; idx += 128) {
    const int r = idx / CH, c = idx % CH;
    const int row = mt * ROWS + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < M && r < ROWS) {
      const int j = row / G, g = row % G;
      v = *reinterpret_cast<const uint4*>(a.q + (q_base + j) * a.q_stride + (kvh * G + g) * D + c * 8);
    }
    *reinterpret_cast<uint4*>(sq + tile_off<D>(r, c)) = v;
  }
  __syncthreads();

  // ---- this CTA's KV range: only what the rows of this tile may see (causal) ----
  const int j_max = min((mt * ROWS + ROWS - 1) / G, q_len - 1);
  const int visible = max(0, kv_len - q_len + 1 + j_max);
  const int per_split = ((visible + a.splits - 1) / a.splits + TOK * 4 - 1) / (TOK * 4) * (TOK * 4);
  const int kv_begin = split * per_split;
  const int kv_end = min(visible, kv_begin + per_split);
  const int n_tiles = kv_end > kv_begin ? (kv_end - kv_begin + TOK - 1) / TOK : 0;

  uint8_t* my = swarp + warp * Cfg::WARP_REGION;
  const int* pt = a.page_table + static_cast<size_t>(b) * a.max_pages;
  const uint32_t ps_mask = static_cast<uint32_t>(a.page_size - 1);

  // Per-lane constants of the load path. A row of K plus the same row of V is PER_ROW
  // 16-byte chunks; with PER_ROW <= 32 a warp issues ROWS_PER_IT whole rows per instruction.
  constexpr int PER_ROW = 2 * CH;
  constexpr int ROWS_PER_IT = PER_ROW <= 32 ? 32 / PER_ROW : 1;
  const int ld_rsub = PER_ROW <= 32 ? lane / PER_ROW : 0;
  const int ld_c2 = PER_ROW <= 32 ? lane % PER_ROW : lane;
  const bool ld_is_v = PER_ROW <= 32 ? (ld_c2 >= CH) : false;
  const int ld_c = ld_is_v ? ld_c2 - CH : ld_c2;
  const size_t row_stride_bytes = static_cast<size_t>(a.Hkv) * D * 2;
  const char* ld_gbase = reinterpret_cast<const char*>(ld_is_v ? a.v_cache : a.k_cache) +
                         (static_cast<size_t>(kvh) * D + ld_c * 8) * 2;
  const uint32_t ld_sbase = smem_u32(my) + (ld_is_v ? TILE_BYTES : 0);

  // One tile = 16 rows of K and of V. Lane r (< 16) resolves row r's cache slot once; the
  // warp then issues whole rows, one 16-byte chunk per lane.
  // Cache slot of row `lane` of a tile (lanes >= 16 and rows past kv_end: -1). Issued one tile
  // ahead of its use, so the page-table load is off the critical path.
  auto resolve_slot = [&](int tile) -> int {
    int my_slot = -1;
    if (lane < TOK && tile < n_tiles) {
      const int t = kv_begin + tile * TOK + lane;
      if (t < kv_end) {
        const int page = pt[t >> a.page_shift];
        const long sl = static_cast<long>(page) * a.page_size + (t & ps_mask);
        if (sl < 0 || sl >= a.cache_slots) set_status(a.status, kStatusBadExtent);
        else my_slot = static_cast<int>(sl);
      }
    }
    return my_slot;
  };
  auto load_tile = [&](int stage, int my_slot) {
    const uint32_t sstage = ld_sbase + stage * 2 * TILE_BYTES;
    if constexpr (PER_ROW <= 32) {
#pragma unroll
      for (int r0 = 0; r0 < TOK; r0 += ROWS_PER_IT) {
        const int r = r0 + ld_rsub;
        const int slot = __shfl_sync(0xffffffffu, my_slot, r);
        const uint32_t dst = sstage + tile_off<D>(r, ld_c);
        if (slot >= 0) {
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst),
                       "l"(ld_gbase + static_cast<size_t>(slot) * row_stride_bytes) : "memory");
        } else {
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dst), "r"(0) : "memory");
        }
      }
    } else {
#pragma unroll 4
      for (int r = 0; r < TOK; ++r) {
        const int slot = __shfl_sync(0xffffffffu, my_slot, r);
        const uint32_t dk = sstage + tile_off<D>(r, ld_c);
        if (slot >= 0) {
          const char* g = ld_gbase + static_cast<size_t>(slot) * row_stride_bytes;
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dk), "l"(g) : "memory");
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dk + TILE_BYTES),
                       "l"(g + (reinterpret_cast<const char*>(a.v_cache) - reinterpret_cast<const char*>(a.k_cache)))
                       : "memory");
        } else {
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dk), "r"(0) : "memory");
          asm volatile("st.shared.v4.u32 [%0], {%1, %1, %1, %1};" ::"r"(dk + TILE_BYTES), "r"(0) : "memory");
        }
      }
    }
  };

  // prologue: fill STAGES-1 stages
  int next_tile = warp;
#pragma unroll
  for (int s = 0; s < Cfg::STAGES - 1; ++s) {
    if (next_tile < n_tiles) load_tile(s, resolve_slot(next_tile));
    cp_async_commit();
    next_tile += 4;
  }
  int slot_ahead = resolve_slot(next_tile);

  // The products are computed transposed so that the query rows (8 per n-tile: exactly one
  // GQA group of 8 heads) sit on the MMA N side and no tensor work is spent on padding:
  //   S^T[tok, qrow] = K[tok, :] . Q[qrow, :]        (A = K tile, B = Q^T)
  //   O^T[d,  qrow] += V^T[d, tok] . P^T[tok, qrow]   (A = V^T via ldmatrix.trans, B = P^T)
  const uint32_t sqa = smem_u32(sq);
  uint32_t qb[Q_REGS ? KT : 1][4];
  if constexpr (Q_REGS) {
#pragma unroll
    for (int ks = 0; ks < KT; ++ks) {
      const int mat = lane >> 3;
      const int row = (mat >> 1) * 8 + (lane & 7);
      ldsm_x4(sqa + tile_off<D>(row, ks * 2 + (mat & 1)), qb[ks][0], qb[ks][1], qb[ks][2], qb[ks][3]);
    }
  }

  float ot[D / 16][NQ][4];
#pragma unroll
  for (int i = 0; i < D / 16; ++i)
#pragma unroll
    for (int n = 0; n < NQ; ++n) ot[i][n][0] = ot[i][n][1] = ot[i][n][2] = ot[i][n][3] = 0.f;
  // per-thread columns: qrow = n*8 + 2*(lane%4) + c, c in {0,1}
  float m_run[NQ][2], l_run[NQ][2];
  int lim[NQ][2];
#pragma unroll
  for (int n = 0; n < NQ; ++n)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      m_run[n][c] = -INFINITY;
      l_run[n][c] = 0.f;
      const int row = mt * ROWS + n * 8 + (lane & 3) * 2 + c;
      const int j = row < M ? row / G : 0;
      lim[n][c] = row < M ? kv_len - q_len + 1 + j : 0;
    }

  // Smallest causal limit among the valid rows of this CTA, never past kv_end. Padding rows
  // hold q = 0 and are never written, so a tile below this limit needs no masking at all.
  const int first_row = mt * ROWS;
  const int min_lim = first_row < M ? min(kv_end, kv_len - q_len + 1 + first_row / G) : kv_end;
  int stage = 0;
  for (int tile = warp; tile < n_tiles; tile += 4) {
    {
      int ls = stage + Cfg::STAGES - 1;
      if (ls >= Cfg::STAGES) ls -= Cfg::STAGES;
      if (next_tile < n_tiles) load_tile(ls, slot_ahead);
      cp_async_commit();
      next_tile += 4;
      slot_ahead = resolve_slot(next_tile);
    }
    cp_async_wait<Cfg::STAGES - 1>();
    __syncwarp();
    const uint32_t sk = smem_u32(my + stage * 2 * TILE_BYTES);
    const uint32_t sv = sk + TILE_BYTES;

    float st[NQ][4];
#pragma unroll
    for (int n = 0; n < NQ; ++n) st[n][0] = st[n][1] = st[n][2] = st[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < KT; ++ks) {
      uint32_t ka[4];
      {
        const int mat = lane >> 3;
        const int row = (mat & 1) * 8 + (lane & 7);
        ldsm_x4(sk + tile_off<D>(row, ks * 2 + (mat >> 1)), ka[0], ka[1], ka[2], ka[3]);
      }
      uint32_t q0, q1, q2, q3;
      if constexpr (Q_REGS) {
        q0 = qb[ks][0]; q1 = qb[ks][1]; q2 = qb[ks][2]; q3 = qb[ks][3];
      } else {
        const int mat = lane >> 3;
        const int row = (mat >> 1) * 8 + (lane & 7);
        ldsm_x4(sqa + tile_off<D>(row, ks * 2 + (mat & 1)), q0, q1, q2, q3);
      }
      mma_bf16_16816(st[0], ka, q0, q1);
      if constexpr (NQ == 2) mma_bf16_16816(st[1], ka, q2, q3);
    }
    // ---- mask + online softmax over the token (row) dimension ----
    const int t0 = kv_begin + tile * TOK;
    const bool full_tile = t0 + TOK <= min_lim;      // every row of the CTA sees the whole tile
    uint32_t pb[NQ][2];
#pragma unroll
    for (int n = 0; n < NQ; ++n) {
      float corr[2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        // elements of column c: st[n][c] (token lane/4) and st[n][c + 2] (token lane/4 + 8)
        float mx = -INFINITY;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = t0 + (lane >> 2) + h * 8;
          float v = st[n][c + 2 * h] * a.scale_log2;
          if (!full_tile && (t >= lim[n][c] || t >= kv_end)) v = -INFINITY;
          st[n][c + 2 * h] = v;
          mx = fmaxf(mx, v);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float m_new = fmaxf(m_run[n][c], mx);
        corr[c] = (m_new == -INFINITY) ? 1.f : fast_exp2(m_run[n][c] - m_new);
        m_run[n][c] = m_new;
        float lsum = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float p = (m_new == -INFINITY) ? 0.f : fast_exp2(st[n][c + 2 * h] - m_new);
          st[n][c + 2 * h] = p;
          lsum += p;
        }
        l_run[n][c] = l_run[n][c] * corr[c] + lsum;
      }
      if (__any_sync(0xffffffffu, corr[0] != 1.f || corr[1] != 1.f)) {
#pragma unroll
        for (int i = 0; i < D / 16; ++i) {
          ot[i][n][0] *= corr[0];
          ot[i][n][1] *= corr[1];
          ot[i][n][2] *= corr[0];
          ot[i][n][3] *= corr[1];
        }
      }
      // P^T as the B operand: transpose the two 8x8 blocks (tokens 0-7, 8-15) in registers
      pb[n][0] = movmatrix_trans(pack_bf16(st[n][0], st[n][1]));
      pb[n][1] = movmatrix_trans(pack_bf16(st[n][2], st[n][3]));
    }
    // ---- O^T += V^T P^T ----
#pragma unroll
    for (int dt = 0; dt < D / 16; ++dt) {
      uint32_t va[4];
      const int mat = lane >> 3;
      const int row = (mat >> 1) * 8 + (lane & 7);
      ldsm_x4_t(sv + tile_off<D>(row, dt * 2 + (mat & 1)), va[0], va[1], va[2], va[3]);
      mma_bf16_16816(ot[dt][0], va, pb[0][0], pb[0][1]);
      if constexpr (NQ == 2) mma_bf16_16816(ot[dt][1], va, pb[1][0], pb[1][1]);
    }
    __syncwarp();
    if (++stage == Cfg::STAGES) stage = 0;
  }
  cp_async_wait<0>();
#pragma unroll
  for (int n = 0; n < NQ; ++n)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      l_run[n][c] += __shfl_xor_sync(0xffffffffu, l_run[n][c], 4);
      l_run[n][c] += __shfl_xor_sync(0xffffffffu, l_run[n][c], 8);
      l_run[n][c] += __shfl_xor_sync(0xffffffffu, l_run[n][c], 16);
    }

  // ---- merge the 4 warps through shared memory (each warp reuses its own ring) ----
  __syncwarp();
  float* wo = reinterpret_cast<float*>(my);          // [16][D]
  float* wm = wo + 16 * D;                           // [16]
  float* wl = wm + 16;                               // [16]
#pragma unroll
  for (int dt = 0; dt < D / 16; ++dt)
#pragma unroll
    for (int n = 0; n < NQ; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qrow = n * 8 + (lane & 3) * 2 + (e & 1);
        const int d = dt * 16 + (lane >> 2) + (e >> 1) * 8;
        wo[qrow * D + d] = ot[dt][n][e];
      }
  if ((lane >> 2) == 0) {
#pragma unroll
    for (int n = 0; n < NQ; ++n)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int qrow = n * 8 + (lane & 3) * 2 + c;
        wm[qrow] = m_run[n][c];
        wl[qrow] = l_run[n][c];
      }
  }
  __syncthreads();
  const size_t tile_id = (static_cast<size_t>(b) * a.Hkv + kvh) * a.m_tiles + mt;
  // Per-row weights of the four warps, computed once: f[w][r] = 2^(m_w - m) / l, and the
  // row's log-sum-exp for the split merge.
  __shared__ float s_f[4][16];
  __shared__ float s_lse[16];
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    float mw[4], mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      mw[w] = reinterpret_cast<float*>(swarp + w * Cfg::WARP_REGION)[16 * D + r];
      mm = fmaxf(mm, mw[w]);
    }
    float l = 0.f, f[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      f[w] = (mw[w] == -INFINITY) ? 0.f : exp2f(mw[w] - mm);
      l += reinterpret_cast<float*>(swarp + w * Cfg::WARP_REGION)[16 * D + 16 + r] * f[w];
    }
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) s_f[w][r] = f[w] * inv;
    s_lse[r] = l > 0.f ? mm + log2f(l) : -INFINITY;
  }
  __syncthreads();
  constexpr int D4 = D / 4;
  for (int idx = threadIdx.x; idx < ROWS * D4; idx += 128) {
    const int r = idx / D4, d = (idx % D4) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float4 v = *reinterpret_cast<const float4*>(reinterpret_cast<float*>(swarp + w * Cfg::WARP_REGION) + r * D + d);
      const float f = s_f[w][r];
      acc.x += v.x * f; acc.y += v.y * f; acc.z += v.z * f; acc.w += v.w * f;
    }
    const int row = mt * ROWS + r;
    if (a.splits == 1) {
      if (row < M) {
        const int j = row / G, g = row % G;
        uint2 o;
        o.x = pack_bf16(acc.x, acc.y);
        o.y = pack_bf16(acc.z, acc.w);
        *reinterpret_cast<uint2*>(a.out + ((q_base + j) * a.Hq + kvh * G + g) * D + d) = o;
      }
    } else {
      const size_t pidx = tile_id * a.splits + split;
      *reinterpret_cast<float4*>(a.part_o + (pidx * 16 + r) * D + d) = acc;
      if (d == 0) a.part_lse[pidx * 16 + r] = s_lse[r];
    }
  }
  if (a.splits == 1) return;

  // ---- the last split CTA of this (request, kv head, row tile) merges the splits ----
  __shared__ int s_last;
  __shared__ float s_w[kMaxSplits][16];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(a.part_count + tile_id, 1u);
    s_last = (prev == static_cast<unsigned int>(a.splits) - 1u);
    if (s_last) a.part_count[tile_id] = 0;     // ready for the next launch
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const size_t p0 = tile_id * a.splits;
  // every (split, row) log-sum-exp is fetched by its own thread, so the loads overlap
  for (int idx = threadIdx.x; idx < a.splits * 16; idx += 128)
    s_w[idx >> 4][idx & 15] = __ldcg(a.part_lse + p0 * 16 + idx);
  __syncthreads();
  if (threadIdx.x < 16) {
    const int r = threadIdx.x;
    float mm = -INFINITY;
    for (int s2 = 0; s2 < a.splits; ++s2) mm = fmaxf(mm, s_w[s2][r]);
    float wsum = 0.f;
    for (int s2 = 0; s2 < a.splits; ++s2) {
      const float lse = s_w[s2][r];
      const float w = (lse == -INFINITY) ? 0.f : exp2f(lse - mm);
      s_w[s2][r] = w;
      wsum += w;
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    for (int s2 = 0; s2 < a.splits; ++s2) s_w[s2][r] *= inv;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < ROWS * D4; idx += 128) {
    const int r = idx / D4, d = (idx % D4) * 4;
    const int row = mt * ROWS + r;
    if (row >= M) continue;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* src = a.part_o + (p0 * 16 + r) * D + d;
#pragma unroll 4
    for (int s2 = 0; s2 < a.splits; ++s2) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src + static_cast<size_t>(s2) * 16 * D));
      const float w = s_w[s2][r];
      acc.x += v.x * w; acc.y += v.y * w; acc.z += v.z * w; acc.w += v.w * w;
    }
    const int j = row / G, g = row % G;
    uint2 o;
    o.x = pack_bf16(acc.x, acc.y);
    o.y = pack_bf16(acc.z, acc.w);
    *reinterpret_cast<uint2*>(a.out + ((q_base + j) * a.Hq + kvh * G + g) * D + d) = o;
  }
}

template <int D, int NQ>
static int launch_decode_nq(const DecodeAttnArgs& a, cudaStream_t st) {
  using Cfg = AttnCfg<D>;
  auto kern = decode_attn_kernel<D, NQ>;
  static bool set = false;
  if (!set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
    if (e != cudaSuccess) return static_cast<int>(e);
    set = true;
  }
  dim3 grid(a.splits, a.Hkv * a.m_tiles, a.B);
  cudaError_t le = launch_pdl(kern, grid, dim3(128), Cfg::SMEM, st, 1, a);
  if (le != cudaSuccess) return static_cast<int>(le);
  return 0;
}

template <int D>
static int launch_decode(const DecodeAttnArgs& a, cudaStream_t st) {
  const int M = (a.Hq / a.Hkv) * a.q_len;
  return M <= 8 ? launch_decode_nq<D, 1>(a, st) : launch_decode_nq<D, 2>(a, st);
}

}  // namespace afd

// Split-KV workspace layout, in bytes from the start:
//   [0, kCounterRegionBytes)   one arrival counter per (request, kv head, row tile); they must be
//                              zero when a launch starts and every launch leaves them zero again
//   then part_o  [tiles][16][D] fp32, then part_lse [tiles][16] fp32
// The counters sit in FRONT of the partials at an offset that does not depend on (B, splits), so a
// workspace that is zeroed once can be shared by launches of any shape: a later launch never finds
// its counters on top of an earlier launch's partial results.
static constexpr long kCounterRegionBytes = 256 * 1024;

extern "C" long afd_decode_attn_workspace_bytes(int B, int Hq, int Hkv, int q_len, int D, int splits) {
  const int G = Hq / Hkv;
  const long m_tiles = (G * q_len + 15) / 16;
  const long tiles = static_cast<long>(B) * Hkv * m_tiles * splits;
  return kCounterRegionBytes + tiles * 16 * D * 4 + tiles * 16 * 4;
}

extern "C" int afd_decode_attention_strided(const void* q, long q_stride, const void* k_cache,
                                            const void* v_cache, const void* page_table,
                                            const void* seq_lens, void* out, void* workspace, int B,
                                            int Hq, int Hkv, int D, int q_len, int page_size,
                                            int max_pages, long cache_slots, int splits, float sm_scale,
                                            void* status, void* stream);

extern "C" int afd_decode_attention(const void* q, const void* k_cache, const void* v_cache,
                                    const void* page_table, const void* seq_lens, void* out,
                                    void* workspace, int B, int Hq, int Hkv, int D, int q_len,
                                    int page_size, int max_pages, long cache_slots, int splits,
                                    float sm_scale, void* status, void* stream) {
  return afd_decode_attention_strided(q, static_cast<long>(Hq) * D, k_cache, v_cache, page_table, seq_lens, out,
                                      workspace, B, Hq, Hkv, D, q_len, page_size, max_pages, cache_slots, splits,
                                      sm_scale, status, stream);
}

static int launch_attention(const void* q, long q_stride, const void* k_cache, const void* v_cache,
                            const void* page_table, const void* seq_lens, const void* q_starts, void* out,
                            void* workspace, int B, int Hq, int Hkv, int D, int q_len, int page_size, int max_pages,
                            long cache_slots, int splits, float sm_scale, void* status, void* stream);

// Same, with q rows `q_stride` elements apart (q read in place from a merged qkv buffer).
extern "C" int afd_decode_attention_strided(const void* q, long q_stride, const void* k_cache,
                                            const void* v_cache, const void* page_table,
                                            const void* seq_lens, void* out, void* workspace, int B,
                                            int Hq, int Hkv, int D, int q_len, int page_size,
                                            int max_pages, long cache_slots, int splits, float sm_scale,
                                            void* status, void* stream) {
  return launch_attention(q, q_stride, k_cache, v_cache, page_table, seq_lens, nullptr, out, workspace, B, Hq, Hkv, D,
                          q_len, page_size, max_pages, cache_slots, splits, sm_scale, status, stream);
}

// Causal attention of the new chunk of every request against its paged KV in ONE launch: request b
// owns the query rows [q_starts[b], q_starts[b + 1]) (chunks of different lengths, `max_q_len` the
// longest) and sees the first seq_lens[b] - chunk_len + 1 + j cached tokens from its j-th row.
extern "C" int afd_prefill_attention_varlen(const void* q, long q_stride, const void* k_cache, const void* v_cache,
                                            const void* page_table, const void* seq_lens, const void* q_starts,
                                            void* out, int B, int Hq, int Hkv, int D, int max_q_len, int page_size,
                                            int max_pages, long cache_slots, float sm_scale, void* status,
                                            void* stream) {
  if (q_starts == nullptr || max_q_len < 1) return -8;
  return launch_attention(q, q_stride, k_cache, v_cache, page_table, seq_lens, q_starts, out, nullptr, B, Hq, Hkv, D,
                          max_q_len, page_size, max_pages, cache_slots, 1, sm_scale, status, stream);
}

static int launch_attention(const void* q, long q_stride, const void* k_cache, const void* v_cache,
                            const void* page_table, const void* seq_lens, const void* q_starts, void* out,
                            void* workspace, int B, int Hq, int Hkv, int D, int q_len, int page_size, int max_pages,
                            long cache_slots, int splits, float sm_scale, void* status, void* stream) {
  using namespace afd;
  if (B == 0) return 0;
  if (Hq % Hkv != 0 || splits < 1 || splits > afd::kMaxSplits || page_size < 1) return -1;
  if (splits > 1 && workspace == nullptr) return -2;
  DecodeAttnArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.q_stride = q_stride;
  if (q_stride % 8 != 0) return -5;
  a.k_cache = static_cast<const __nv_bfloat16*>(k_cache);
  a.v_cache = static_cast<const __nv_bfloat16*>(v_cache);
  a.page_table = static_cast<const int*>(page_table);
  a.seq_lens = static_cast<const int*>(seq_lens);
  a.q_starts = static_cast<const int*>(q_starts);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.B = B; a.Hq = Hq; a.Hkv = Hkv; a.q_len = q_len; a.page_size = page_size; a.max_pages = max_pages;
  a.splits = splits;
  a.m_tiles = ((Hq / Hkv) * q_len + 15) / 16;
  a.cache_slots = cache_slots;
  a.scale_log2 = sm_scale * 1.4426950408889634f;
  a.status = static_cast<int*>(status);
  const long tiles = static_cast<long>(B) * Hkv * a.m_tiles * splits;
  if (static_cast<long>(Hkv) * a.m_tiles > 65535 || B > 65535) return -9;      // grid y / z limits
  if (splits > 1 && static_cast<long>(B) * Hkv * a.m_tiles * 4 > kCounterRegionBytes) return -7;
  a.part_count = static_cast<unsigned int*>(workspace);
  a.part_o = workspace ? reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterRegionBytes) : nullptr;
  a.part_lse = a.part_o ? a.part_o + tiles * 16 * D : nullptr;
  if ((page_size & (page_size - 1)) != 0) return -4;
  if (cache_slots > 0x7fffffffL) return -6;     // page sizes are powers of two
  a.page_shift = 0;
  while ((1 << a.page_shift) < page_size) ++a.page_shift;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (D == 128) return launch_decode<128>(a, st);
  if (D == 256) return launch_decode<256>(a, st);
  if (D == 64) return launch_decode<64>(a, st);
  return -3;
}
