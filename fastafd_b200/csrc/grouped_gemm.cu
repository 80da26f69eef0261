// Expert-grouped GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), the
// compute core of the MLP-server (expert GPU) side and of the dense projections.
//
//   out[row, n] = sum_k X[row, k] * W[e(row), n, k]
//
// Weights sit on the UMMA M side (128 weight rows per tile) and tokens on the UMMA
// N side (BLOCK_TOK tokens per tile, 16..128), so a decode-sized token group does
// not waste tensor work: the kernel streams each expert's weights once and is
// bound by HBM. Operands arrive by TMA (128-byte swizzle) into a multi-stage
// shared-memory ring; one elected thread issues tcgen05.mma; the accumulator lives
// in TMEM (two stages) and four epilogue warps read it back with tcgen05.ld.
//
// Precision modes:
//   bf16 : kind::f16, one accumulation over the whole K.
//   fp8  : e4m3 operands (kind::f8f6f4) with 128x128 weight block scales and 1x128
//          activation group scales. Each 128-deep K block is accumulated in TMEM
//          on its own and promoted into fp32 registers with the exact product of
//          both scales, so no scale is re-rounded.
//
// Epilogues:
//   STORE   : out[row, n] bf16 (dense projections, tests).
//   SWIGLU  : weight rows are interleaved gate/up in groups of 16 (rows 32b..32b+15
//             = gate features 16b.., rows 32b+16..32b+31 = up features 16b..);
//             out[row, f] = silu(gate) * up, bf16 (or e4m3 + 1x128 scales in fp8
//             mode, where one CTA covers two adjacent tiles = 128 features).
//   COMBINE : the down projection. Each row is stored straight into the attention
//             GPU that owns the token, at combine[k][token][n] in that GPU's
//             memory (peer pointer), and the last CTA to finish releases one flag
//             per attention GPU: GEMM and M2N transfer are one kernel.
//
// The role of the reference's expert-GPU megakernel (L1/L2 grouped GEMMs with
// SwiGLU and remote combine stores) is described in
// python/minisgl/kernel/csrc/deepgemm/deep_gemm/include/deep_gemm/impls/sm100_mega_moe_m2n.cuh:1270-3073;
// this file is an independent design (1-CTA tiles, exact block scales, push flags).
#include "common.cuh"

namespace afd {

enum Epilogue : int { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_COMBINE = 2 };

constexpr int kMaxPeers = 16;

struct GroupedGemmArgs {
  // Tile schedule written by the grouping kernel: tile_info[t] = {expert, row_start,
  // valid_rows, 0} for token tile t; *num_tok_tiles of them.
  const int4* tile_info;
  const int* num_tok_tiles;
  int max_tok_tiles;
  int n_tiles;    // weight rows per expert / 128
  int k_blocks;   // K / 64 (bf16) or K / 128 (fp8)
  int n_per_expert;  // weight rows per expert
  int out_ld;     // leading dimension of out (elements)
  int pool_rows;  // rows in X / out pools (bounds check)
  __nv_bfloat16* out;        // STORE / SWIGLU (bf16 mode)
  // fp8 mode
  const float* x_scale;      // [pool_rows][k_blocks]
  const float* w_scale;      // [E][n_tiles][2][k_blocks] (per tile half: lanes&16)
  uint8_t* out_q;            // SWIGLU fp8 output [pool_rows][out_ld] e4m3
  float* out_scale;          // SWIGLU fp8 output scales [pool_rows][out_ld/128]
  // COMBINE
  const uint32_t* row_meta;  // [pool_rows]: src<<24 | k<<16 | token
  __nv_bfloat16* peer_combine[kMaxPeers];  // combine buffer base in each attention GPU
  uint32_t* peer_flag[kMaxPeers];          // flag word in each attention GPU (this EG's slot)
  int num_peers;
  int combine_tokens;        // T capacity of combine[k][T][H]
  int hidden;                // H of combine rows
  uint32_t* epoch;           // device word: value to publish, then incremented (COMBINE)
  unsigned int* done_counter;  // device word for the last-CTA election (COMBINE), starts 0
  int* status;
  unsigned long long* trace;   // optional timeline ring (COMBINE: event 3 = flags released)
  // STORE only: split-K. Each work unit covers k_blocks / k_splits of the K blocks and writes an fp32
  // partial tile; the unit that arrives last at the tile's counter sums the partials and stores the
  // tile. Decode-sized dense projections have too few (token tile, weight tile) pairs to fill the GPU
  // otherwise. Counters are zero between launches (the last arriver resets its counter).
  // Weights stored tile by tile: [row tile][k block][128 rows][128 bytes], so that one TMA box
  // (a 128 x 128-byte weight tile) is 16 KB of consecutive memory instead of 128 pieces a whole
  // weight row apart. The tensor map is then [(tiles) * 128][128 bytes] and the box's y coordinate is
  // (row_tile * k_blocks + kb) * 128.
  int w_tile_major;
  int k_splits;
  float* splitk_ws;            // [tok_tiles * n_tiles][k_splits][BLOCK_TOK][128]
  unsigned int* splitk_cnt;    // [tok_tiles * n_tiles]
  const __nv_bfloat16* bias;   // STORE only: optional [n_per_expert], added to every row
  // While the kernel waits for its predecessor (programmatic dependent launch) HBM is idle and the
  // CTAs are resident. Each CTA then pulls the weights of the work unit it will most likely run first
  // into L2: the unit it would get if token tile t held expert t (true when every expert has between
  // one and block_tok tokens, the common case in decode). A hint only: a wrong guess costs bandwidth,
  // never correctness. l2_prefetch_bytes = bytes per CTA (0: off).
  int l2_prefetch_bytes;
  int num_experts;
};

template <int BLOCK_TOK, bool FP8>
struct GemmCfg {
  static constexpr int kWBytes = 128 * 128;              // weight tile per stage
  static constexpr int kXBytes = BLOCK_TOK * 128;        // token tile per stage
  static constexpr int kXBytesPadded = (kXBytes + 1023) / 1024 * 1024;
  static constexpr int kStageBytes = kWBytes + kXBytesPadded;
  static constexpr int kEpiBytes = BLOCK_TOK * (128 + 8) * 2 + (FP8 ? BLOCK_TOK * 64 * 4 : 0);
  static constexpr int kStages = (200 * 1024 - kEpiBytes) / kStageBytes > 10
                                     ? 10
                                     : (200 * 1024 - kEpiBytes) / kStageBytes;
  static constexpr int kSmemBytes = kStages * kStageBytes + kEpiBytes + 1024 /*align*/ + 256;
  static constexpr int kTmemCols = (2 * BLOCK_TOK <= 32) ? 32
                                   : (2 * BLOCK_TOK <= 64) ? 64
                                   : (2 * BLOCK_TOK <= 128) ? 128
                                   : (2 * BLOCK_TOK <= 256) ? 256 : 512;
  static constexpr int kUmmaPerBlock = 4;   // 128 B of K per stage: 4 x (K=16 bf16 | K=32 fp8)
};

__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int BLOCK_TOK, bool FP8, int EPI>
__global__ void __launch_bounds__(192, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_x, const GroupedGemmArgs args) {
  using Cfg = GemmCfg<BLOCK_TOK, FP8>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint8_t* epi_smem = smem + Cfg::kStages * Cfg::kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + Cfg::kEpiBytes);
  uint64_t* full_bar = bars;
  uint64_t* empty_bar = bars + Cfg::kStages;
  uint64_t* tfull_bar = bars + 2 * Cfg::kStages;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  pdl_trigger();       // the next kernel may set itself up while this one streams the weights
  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull_bar[s], 1);
      mbar_init(&tempty_bar[s], 4);
    }
    *abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (args.l2_prefetch_bytes > 0 && warp == 0) {
    // Same boxes as the producer's later loads of the guessed unit, as TMA prefetches into L2.
    constexpr int kTPU = (FP8 && EPI == EPI_SWIGLU) ? 2 : 1;
    const int units_per_tile = args.n_tiles / kTPU;
    const int guess_expert = static_cast<int>(blockIdx.x) / units_per_tile;
    const int guess_unit = static_cast<int>(blockIdx.x) - guess_expert * units_per_tile;
    if (guess_expert < args.num_experts && elect_one()) {
      int boxes = args.l2_prefetch_bytes / Cfg::kWBytes;
      for (int sub = 0; sub < kTPU && boxes > 0; ++sub) {
        const int w_row = guess_expert * args.n_per_expert + (guess_unit * kTPU + sub) * 128;
        for (int kb = 0; kb < args.k_blocks && boxes > 0; ++kb, --boxes) tma_prefetch_2d(&tmap_w, kb * (FP8 ? 128 : 64), w_row);
      }
    }
  }
  pdl_wait();          // barriers, TMEM and descriptors are ready; now the predecessor's outputs may be read
  int num_tok_tiles = *args.num_tok_tiles;
  if (num_tok_tiles > args.max_tok_tiles) {
    if (threadIdx.x == 0) set_status(args.status, kStatusCapacity);
    num_tok_tiles = args.max_tok_tiles;
  }
  // In fp8 SWIGLU mode a CTA owns two adjacent weight tiles (128 features) so that
  // it can compute the 1x128 activation scale; the work unit is then a tile pair.
  constexpr int kTilesPerUnit = (FP8 && EPI == EPI_SWIGLU) ? 2 : 1;
  const int n_units = args.n_tiles / kTilesPerUnit;
  const int ks_n = (EPI == EPI_STORE && args.k_splits > 1) ? args.k_splits : 1;
  const int total_units = num_tok_tiles * n_units * ks_n;
  const int k_blocks = args.k_blocks;
  const int kb_per = k_blocks / ks_n;       // K blocks of one unit (whole K unless split)

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        const int ks = u % ks_n, uu = u / ks_n;
        const int tok_tile = uu / n_units;
        const int unit = uu - tok_tile * n_units;
        const int4 ti = args.tile_info[tok_tile];
        for (int sub = 0; sub < kTilesPerUnit && ok; ++sub) {
          const int n_tile = unit * kTilesPerUnit + sub;
          const int w_row = ti.x * args.n_per_expert + n_tile * 128;
          for (int kb = ks * kb_per; kb < (ks + 1) * kb_per; ++kb) {
            if (!mbar_wait(&empty_bar[stage], phase ^ 1u, abort_flag, args.status)) {
              ok = false;
              break;
            }
            uint8_t* sw = smem + stage * Cfg::kStageBytes;
            uint8_t* sx = sw + Cfg::kWBytes;
            mbar_expect_tx(&full_bar[stage], Cfg::kWBytes + Cfg::kXBytes);
            const int kx = kb * (FP8 ? 128 : 64);
            if (args.w_tile_major) tma_load_2d(sw, &tmap_w, &full_bar[stage], 0, ((w_row >> 7) * k_blocks + kb) * 128);
            else tma_load_2d(sw, &tmap_w, &full_bar[stage], kx, w_row);
            tma_load_2d(sx, &tmap_x, &full_bar[stage], kx, ti.y);
            if (++stage == Cfg::kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      const uint32_t idesc = FP8 ? umma_idesc_e4m3(BLOCK_TOK) : umma_idesc_bf16(BLOCK_TOK);
      int stage = 0;
      uint32_t phase = 0;
      int as = 0;
      uint32_t aphase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
        for (int sub = 0; sub < kTilesPerUnit && ok; ++sub) {
          if (!FP8) {
            if (!mbar_wait(&tempty_bar[as], aphase ^ 1u, abort_flag, args.status)) { ok = false; break; }
            tc_fence_after();
          }
          for (int kb = 0; kb < kb_per; ++kb) {      // relative index: only "first block of the unit" matters here
            if (FP8) {
              if (!mbar_wait(&tempty_bar[as], aphase ^ 1u, abort_flag, args.status)) { ok = false; break; }
              tc_fence_after();
            }
            if (!mbar_wait(&full_bar[stage], phase, abort_flag, args.status)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sw = smem_u32(smem + stage * Cfg::kStageBytes);
            const uint32_t sx = sw + Cfg::kWBytes;
            const uint64_t dw = umma_desc_k128(sw);
            const uint64_t dx = umma_desc_k128(sx);
            const uint32_t tacc = tmem_base + static_cast<uint32_t>(as * BLOCK_TOK);
#pragma unroll
            for (int k = 0; k < Cfg::kUmmaPerBlock; ++k) {
              // +32 bytes of K per step inside the 128-byte swizzle atom (encoded >> 4).
              const uint32_t acc = FP8 ? (k > 0) : ((kb > 0) || (k > 0));
              if (FP8) umma_e4m3(tacc, dw + 2u * k, dx + 2u * k, idesc, acc);
              else     umma_bf16(tacc, dw + 2u * k, dx + 2u * k, idesc, acc);
            }
            tc_commit(&empty_bar[stage]);
            if (++stage == Cfg::kStages) {
              stage = 0;
              phase ^= 1u;
            }
            if (FP8) {
              tc_commit(&tfull_bar[as]);
              as ^= 1;
              if (as == 0) aphase ^= 1u;
            }
          }
          if (!FP8 && ok) {
            tc_commit(&tfull_bar[as]);
            as ^= 1;
            if (as == 0) aphase ^= 1u;
          }
        }
      }
    }
  } else {
    // ---------------- epilogue warps (2..5) ----------------
    const int q = warp & 3;                 // TMEM lane quarter this warp may read
    const int ethread = (warp - 2) * 32 + lane;  // 0..127 within the epilogue group
    __nv_bfloat16* stile = reinterpret_cast<__nv_bfloat16*>(epi_smem);   // [BLOCK_TOK][136]
    float* hbuf = reinterpret_cast<float*>(epi_smem + BLOCK_TOK * 136 * 2);  // fp8: [BLOCK_TOK][64]
    constexpr int kSL = 136;
    volatile int* s_flag = abort_flag + 1;     // split-K: "this unit arrived last" (epilogue warps only)
    int as = 0;
    uint32_t aphase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      const int ks = u % ks_n, uu = u / ks_n;
      const int tok_tile = uu / n_units;
      const int unit = uu - tok_tile * n_units;
      const int4 ti = args.tile_info[tok_tile];
      int valid = ti.z;
      if (valid > BLOCK_TOK) valid = BLOCK_TOK;
      int row0 = ti.y;
      if (row0 < 0 || row0 + valid > args.pool_rows) {
        set_status(args.status, kStatusBadExtent);
        valid = 0;
        row0 = 0;
      }
      for (int sub = 0; sub < kTilesPerUnit && ok; ++sub) {
        const int n_tile = unit * kTilesPerUnit + sub;
        float acc[BLOCK_TOK];
        if (FP8) {
#pragma unroll
          for (int c = 0; c < BLOCK_TOK; ++c) acc[c] = 0.f;
          const float* wsc = args.w_scale +
              ((static_cast<size_t>(ti.x) * args.n_tiles + n_tile) * 2 + ((lane >> 4) & 1)) * k_blocks;
          for (int kb = ks * kb_per; kb < (ks + 1) * kb_per; ++kb) {
            if (!mbar_wait(&tfull_bar[as], aphase, abort_flag, args.status)) { ok = false; break; }
            tc_fence_after();
            const float ws = __ldg(wsc + kb);
            const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(as * BLOCK_TOK);
#pragma unroll
            for (int c0 = 0; c0 < BLOCK_TOK; c0 += 16) {
              float v[16];
              tmem_ld16(taddr + c0, v);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int row = min(row0 + c0 + i, args.pool_rows - 1);
                const float xs = __ldg(args.x_scale + static_cast<size_t>(row) * k_blocks + kb);
                acc[c0 + i] = fmaf(v[i], ws * xs, acc[c0 + i]);
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty_bar[as]);
            as ^= 1;
            if (as == 0) aphase ^= 1u;
          }
          if (!ok) break;
        } else {
          if (!mbar_wait(&tfull_bar[as], aphase, abort_flag, args.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                 static_cast<uint32_t>(as * BLOCK_TOK);
#pragma unroll
          for (int c0 = 0; c0 < BLOCK_TOK; c0 += 16) {
            tmem_ld16(taddr + c0, &acc[c0]);
          }
          tmem_ld_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty_bar[as]);
          as ^= 1;
          if (as == 0) aphase ^= 1u;
        }

        if (EPI == EPI_SWIGLU) {
          // lanes 0..15 hold gate rows, lanes 16..31 the matching up rows.
          const bool upper = (lane & 16) != 0;
          const int feat_in_tile = q * 16 + (lane & 15);       // 0..63
          if (!FP8) {
            const int feat = n_tile * 64 + feat_in_tile;
#pragma unroll
            for (int c = 0; c < BLOCK_TOK; c += 2) {
              const float send = upper ? acc[c] : acc[c + 1];
              const float got = __shfl_xor_sync(0xffffffffu, send, 16);
              // lower lane: token c   -> silu(gate=acc[c]) * up=got
              // upper lane: token c+1 -> silu(gate=got)    * up=acc[c+1]
              const float g = upper ? got : acc[c];
              const float up = upper ? acc[c + 1] : got;
              const int cc = upper ? c + 1 : c;
              if (cc < valid) {
                args.out[static_cast<size_t>(row0 + cc) * args.out_ld + feat] =
                    __float2bfloat16(silu(g) * up);
              }
            }
          } else {
            // stash h (fp32) for this 64-feature half; quantise after both halves.
            epi_bar_sync();   // earlier readers are done with hbuf
#pragma unroll
            for (int c = 0; c < BLOCK_TOK; c += 2) {
              const float send = upper ? acc[c] : acc[c + 1];
              const float got = __shfl_xor_sync(0xffffffffu, send, 16);
              const float g = upper ? got : acc[c];
              const float up = upper ? acc[c + 1] : got;
              const int cc = upper ? c + 1 : c;
              // bf16 rounding of the activation before quantisation (numerics contract)
              const float h = __bfloat162float(__float2bfloat16(silu(g) * up));
              reinterpret_cast<float*>(hbuf)[cc * 64 + feat_in_tile] = h;
            }
            epi_bar_sync();
            // The 1x128 scale needs both halves. hbuf holds the current half; the first
            // half is parked in stile as bf16 (exact: the values are already bf16-rounded).
            if (sub == 0) {
              for (int idx = ethread; idx < BLOCK_TOK * 64; idx += 128) {
                const int c = idx >> 6, f = idx & 63;
                stile[c * kSL + f] = __float2bfloat16(hbuf[c * 64 + f]);
              }
            } else {
              // 4 threads per token, 32 features each (16 from each half).
              for (int c = ethread >> 2; c < BLOCK_TOK; c += 32) {
                const int part = ethread & 3;
                float vals[32];
                float amax = 0.f;
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                  vals[i] = __bfloat162float(stile[c * kSL + part * 16 + i]);
                  vals[16 + i] = hbuf[c * 64 + part * 16 + i];
                  amax = fmaxf(amax, fmaxf(fabsf(vals[i]), fabsf(vals[16 + i])));
                }
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                const float scale = fmaxf(amax, 1e-10f) / 448.f;
                const float inv = 1.f / scale;
                if (c < valid) {
                  const size_t row = static_cast<size_t>(row0 + c);
                  const int f0 = unit * 128;
                  uint8_t* dst = args.out_q + row * args.out_ld + f0;
#pragma unroll
                  for (int i = 0; i < 16; ++i) {
                    dst[part * 16 + i] = static_cast<uint8_t>(
                        __nv_cvt_float_to_fp8(vals[i] * inv, __NV_SATFINITE, __NV_E4M3));
                    dst[64 + part * 16 + i] = static_cast<uint8_t>(
                        __nv_cvt_float_to_fp8(vals[16 + i] * inv, __NV_SATFINITE, __NV_E4M3));
                  }
                  if (part == 0) args.out_scale[row * (args.out_ld / 128) + unit] = scale;
                }
              }
            }
          }
        } else {
          if (EPI == EPI_STORE && ks_n > 1) {
            // split-K: park this unit's fp32 partial; the last unit of the tile sums all of them
            const int tile_id = tok_tile * args.n_tiles + n_tile;
            float* wsp = args.splitk_ws + (static_cast<size_t>(tile_id) * ks_n + ks) * (BLOCK_TOK * 128);
#pragma unroll
            for (int c = 0; c < BLOCK_TOK; ++c) wsp[c * 128 + q * 32 + lane] = acc[c];
            __threadfence();
            epi_bar_sync();
            if (ethread == 0) {
              const unsigned int prev = atomicAdd(args.splitk_cnt + tile_id, 1u);
              const int last = prev == static_cast<unsigned int>(ks_n) - 1u;
              if (last) args.splitk_cnt[tile_id] = 0;
              *s_flag = last;
            }
            epi_bar_sync();
            if (!*s_flag) continue;
            __threadfence();
            const float* wst = args.splitk_ws + static_cast<size_t>(tile_id) * ks_n * (BLOCK_TOK * 128);
#pragma unroll
            for (int c = 0; c < BLOCK_TOK; ++c) acc[c] = 0.f;
            for (int s = 0; s < ks_n; ++s) {
#pragma unroll
              for (int c = 0; c < BLOCK_TOK; ++c) acc[c] += __ldcg(wst + (static_cast<size_t>(s) * BLOCK_TOK + c) * 128 + q * 32 + lane);
            }
          }
          if (EPI == EPI_STORE && args.bias != nullptr) {
            const float bv = __bfloat162float(args.bias[n_tile * 128 + q * 32 + lane]);
#pragma unroll
            for (int c = 0; c < BLOCK_TOK; ++c) acc[c] += bv;
          }
          // STORE / COMBINE: transpose through shared memory so that each warp writes
          // whole 256-byte token rows (8 bytes per lane).
          epi_bar_sync();   // previous tile's readers are done with stile
#pragma unroll
          for (int c = 0; c < BLOCK_TOK; ++c) {
            stile[c * kSL + q * 32 + lane] = __float2bfloat16(acc[c]);
          }
          epi_bar_sync();
          const int ew = warp - 2;
          for (int c = ew; c < valid; c += 4) {
            const uint2 v = *reinterpret_cast<const uint2*>(&stile[c * kSL + lane * 4]);
            const int row = row0 + c;
            if (EPI == EPI_STORE) {
              __nv_bfloat16* dst = args.out + static_cast<size_t>(row) * args.out_ld + n_tile * 128;
              *reinterpret_cast<uint2*>(dst + lane * 4) = v;
            } else {
              const uint32_t meta = args.row_meta[row];
              const int src = meta >> 24, kk = (meta >> 16) & 0xff, tok = meta & 0xffff;
              if (src >= args.num_peers || tok >= args.combine_tokens) {
                set_status(args.status, kStatusBadExtent);
              } else {
                __nv_bfloat16* dst = args.peer_combine[src] +
                    (static_cast<size_t>(kk) * args.combine_tokens + tok) * args.hidden + n_tile * 128;
                *reinterpret_cast<uint2*>(dst + lane * 4) = v;
              }
            }
          }
        }
      }
    }
  }

  // ---------------- teardown ----------------
  if (*abort_flag) {
    // a wait ran out: give bulk copies already issued time to land before smem is released
    for (int i = 0; i < 1000; ++i) __nanosleep(1000);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }

  if (EPI == EPI_COMBINE) {
    // Publish: all of this CTA's peer stores are ordered before the counter bump;
    // the last CTA to bump releases one flag per attention GPU.
    if (threadIdx.x == 0) {
      __threadfence();            // gpu scope per CTA; the last CTA alone issues the system fence
      const unsigned int prev = atomicAdd(args.done_counter, 1u);
      if (prev == gridDim.x - 1) {
        __threadfence_system();
        const uint32_t e = *args.epoch;
        for (int p = 0; p < args.num_peers; ++p) st_relaxed_sys(args.peer_flag[p], e);   // ordered by the fence above
        trace_stamp(args.trace, e, 3);
        *args.epoch = e + 1;
        *args.done_counter = 0;
        __threadfence();
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// Host side: tensor-map construction and launch.
// ---------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qres;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qres) ==
            cudaSuccess && qres == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  }
  return fn;
}

// 2-D row-major [rows][cols] map, box {128 bytes, box_rows}, 128-byte swizzle.
static int make_tmap_2d(CUtensorMap* m, const void* base, int elem_bytes, uint64_t rows,
                        uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (fn == nullptr) return -1;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * static_cast<uint64_t>(elem_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elem_bytes), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, elem_bytes == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                  2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -static_cast<int>(r) - 1000;
}

template <int BLOCK_TOK, bool FP8, int EPI>
static int launch_cfg(const CUtensorMap& tw, const CUtensorMap& tx, const GroupedGemmArgs& a, int grid,
                      cudaStream_t stream) {
  using Cfg = GemmCfg<BLOCK_TOK, FP8>;
  auto kern = grouped_gemm_kernel<BLOCK_TOK, FP8, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return static_cast<int>(e);
    attr_set = true;
  }
  cudaError_t le = launch_pdl(kern, dim3(grid), dim3(192), Cfg::kSmemBytes, stream, 1, tw, tx, a);
  if (le != cudaSuccess) return static_cast<int>(le);
  return 0;
}

template <bool FP8, int EPI>
static int launch_tok(int block_tok, const CUtensorMap& tw, const CUtensorMap& tx, const GroupedGemmArgs& a,
                      int grid, cudaStream_t stream) {
  switch (block_tok) {
    case 16: return launch_cfg<16, FP8, EPI>(tw, tx, a, grid, stream);
    case 32: return launch_cfg<32, FP8, EPI>(tw, tx, a, grid, stream);
    case 64: return launch_cfg<64, FP8, EPI>(tw, tx, a, grid, stream);
    case 128:
      if constexpr (!FP8) return launch_cfg<128, FP8, EPI>(tw, tx, a, grid, stream);
      return -3;
    default: return -2;
  }
}

}  // namespace afd

// C ABI. All pointers are device pointers unless stated. Returns 0 on success, a
// positive cudaError_t, or a negative argument error.
struct AfdGroupedGemmDesc {
  const void* w;          // weights [E * n_per_expert][K] (bf16 or e4m3), K-contiguous
  const void* x;          // token pool [pool_rows][K]
  int num_experts, n_per_expert, k, pool_rows;
  int block_tok, fp8, epilogue, grid;
  const void* tile_info;  // int4[max_tok_tiles]
  const void* num_tok_tiles;
  int max_tok_tiles;
  void* out; int out_ld;
  const void* x_scale; const void* w_scale; void* out_q; void* out_scale;
  const void* row_meta;
  void* peer_combine[afd::kMaxPeers];
  void* peer_flag[afd::kMaxPeers];
  int num_peers, combine_tokens, hidden;
  void* epoch; void* done_counter; void* status; void* trace;
  int k_splits; void* splitk_ws; void* splitk_cnt; const void* bias;
  int w_tile_major;
  int l2_prefetch_bytes;  // total bytes that the CTAs may pull into L2 before the predecessor is done (0: off)
};

extern "C" int afd_grouped_gemm(const AfdGroupedGemmDesc* d, void* stream_v) {
  using namespace afd;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_v);
  const int eb = d->fp8 ? 1 : 2;
  const int kblk = d->fp8 ? 128 : 64;
  if (d->n_per_expert % 128 != 0 || d->k % kblk != 0) return -10;
  if (d->fp8 && d->epilogue == EPI_SWIGLU && (d->n_per_expert / 128) % 2 != 0) return -11;
  if (d->num_peers > kMaxPeers) return -12;
  CUtensorMap tw, tx;
  int r = d->w_tile_major
              ? make_tmap_2d(&tw, d->w, eb, static_cast<uint64_t>(d->num_experts) * d->n_per_expert * (d->k / kblk), kblk, 128)
              : make_tmap_2d(&tw, d->w, eb, static_cast<uint64_t>(d->num_experts) * d->n_per_expert, d->k, 128);
  if (r != 0) return r;
  r = make_tmap_2d(&tx, d->x, eb, d->pool_rows, d->k, d->block_tok);
  if (r != 0) return r;
  GroupedGemmArgs a{};
  a.tile_info = static_cast<const int4*>(d->tile_info);
  a.num_tok_tiles = static_cast<const int*>(d->num_tok_tiles);
  a.max_tok_tiles = d->max_tok_tiles;
  a.n_tiles = d->n_per_expert / 128;
  a.k_blocks = d->k / kblk;
  a.n_per_expert = d->n_per_expert;
  a.out_ld = d->out_ld;
  a.pool_rows = d->pool_rows;
  a.out = static_cast<__nv_bfloat16*>(d->out);
  a.x_scale = static_cast<const float*>(d->x_scale);
  a.w_scale = static_cast<const float*>(d->w_scale);
  a.out_q = static_cast<uint8_t*>(d->out_q);
  a.out_scale = static_cast<float*>(d->out_scale);
  a.row_meta = static_cast<const uint32_t*>(d->row_meta);
  for (int i = 0; i < d->num_peers; ++i) {
    a.peer_combine[i] = static_cast<__nv_bfloat16*>(d->peer_combine[i]);
    a.peer_flag[i] = static_cast<uint32_t*>(d->peer_flag[i]);
  }
  a.num_peers = d->num_peers;
  a.combine_tokens = d->combine_tokens;
  a.hidden = d->hidden;
  a.epoch = static_cast<uint32_t*>(d->epoch);
  a.done_counter = static_cast<unsigned int*>(d->done_counter);
  a.status = static_cast<int*>(d->status);
  a.trace = static_cast<unsigned long long*>(d->trace);
  a.w_tile_major = d->w_tile_major;
  a.k_splits = d->k_splits > 1 ? d->k_splits : 1;
  a.splitk_ws = static_cast<float*>(d->splitk_ws);
  a.splitk_cnt = static_cast<unsigned int*>(d->splitk_cnt);
  a.bias = static_cast<const __nv_bfloat16*>(d->bias);
  a.num_experts = d->num_experts;
  a.l2_prefetch_bytes = (d->l2_prefetch_bytes > 0 && !d->w_tile_major && a.k_splits == 1)
                            ? d->l2_prefetch_bytes / (d->grid > 0 ? d->grid : 148) / 128 * 128 : 0;
  if (a.k_splits > 1 && (d->epilogue != EPI_STORE || a.k_blocks % a.k_splits != 0 || a.splitk_ws == nullptr ||
                         a.splitk_cnt == nullptr))
    return -13;
  if (a.bias != nullptr && d->epilogue != EPI_STORE) return -14;
  const int grid = d->grid > 0 ? d->grid : 148;
  if (d->fp8) {
    switch (d->epilogue) {
      case EPI_STORE: return launch_tok<true, EPI_STORE>(d->block_tok, tw, tx, a, grid, stream);
      case EPI_SWIGLU: return launch_tok<true, EPI_SWIGLU>(d->block_tok, tw, tx, a, grid, stream);
      case EPI_COMBINE: return launch_tok<true, EPI_COMBINE>(d->block_tok, tw, tx, a, grid, stream);
    }
  } else {
    switch (d->epilogue) {
      case EPI_STORE: return launch_tok<false, EPI_STORE>(d->block_tok, tw, tx, a, grid, stream);
      case EPI_SWIGLU: return launch_tok<false, EPI_SWIGLU>(d->block_tok, tw, tx, a, grid, stream);
      case EPI_COMBINE: return launch_tok<false, EPI_COMBINE>(d->block_tok, tw, tx, a, grid, stream);
    }
  }
  return -2;
}
