// Triangle attention around the starting / ending node, fused on sm_100a.
//
// Reference operator: TriangleAttention.forward with the "fireprot" kernel
// (patches/protenix/0002-...patch:35-58, 0005-...patch:19-42), math as in
// python/fireprot/adapters/atlasfold/runtime.py:32-71:
//   x = LN(z) (z^T for the ending node); q,k,v = x W{q,k,v}^T (q * d^-1/2)
//   b^h_jk = x_jk . Wbias_h ; s_ijk = q_ij . k_ik + 1e9 (mask_ik - 1) + b^h_jk
//   o_ij = sum_k softmax_k(s) v_ik ; delta_ij = W_o (sigmoid(x Wg^T + bg) * o) + bo
//   z <- z + delta (ending node: delta transposed back).
//
// Three launches per call, all in "y" coordinates (y = z, or z^T for the
// ending node, addressed through transposed reads; nothing is copied):
//  1. proj: LN + [Wq;Wk;Wv;Wg] GEMM (tcgen05, 128 x 512 per tile) + the
//     4-head pair bias on CUDA cores in FP32; writes q,k as [i][h][j][d], v
//     as [i][h][d][k] (K-major for PV), the gate sigmoid(x Wg^T + b_g) as
//     [i][j][128], bias [h][j][k], mask bias [i][k].
//  2. attn: one CTA per (128 queries, head, row i); key tiles stream by TMA;
//     S = Q K^T in TMEM (double-buffered), online softmax by the 128 row
//     threads (FP32, SFU exp2), P V on tcgen05 into TMEM; the epilogue
//     multiplies o by the gate.
//  3. out: (gate * o) W_o^T (one GEMM) + b_o, residual add in place.
#include "kernels.h"
#include "rowgemm.cuh"

namespace fpb {

constexpr int kHeads = 4;
constexpr int kHeadDim = 32;
constexpr float kMaskInf = 1e9f;

// Pair bias layout, j-blocked: [ceil(n/32)][head][ldb/4][32 rows j][4 keys k]
// (ldb = keys padded to 32). A warp's 32 query rows read 4 keys each as one
// contiguous 512-byte access, and rows [32q, 32q + 32m) form one contiguous
// block (the all-gather unit of the row-sharded path).
__host__ __device__ __forceinline__ size_t bias_index(int j, int h, int k, int ldb) {
  return ((((size_t)(j >> 5) * kHeads + h) * (size_t)(ldb >> 2) + (size_t)(k >> 2)) * 32 +
          (size_t)(j & 31)) * 4 + (size_t)(k & 3);
}
// floats of a pair bias buffer for n rows
__host__ __device__ __forceinline__ size_t bias_elems(int n, int ldb) {
  return (size_t)((n + 31) / 32) * 32 * kHeads * ldb;
}

// ============================================================================
// 1. projection
// ============================================================================
// Pair rows of y: yrows x n (y = z_loc rows, or z^T for the unsharded
// ending node); r0 = global index of local row 0 (pair bias rows, mask).
struct AttnProjArgs {
  const float* z;
  const float* mask;  // nullable, [n][n] global
  int n;
  int yrows;
  int r0;
  float eps;
  const float* ln_w;
  const float* ln_b;
  const float* w_bias;  // [4][128]
  float q_scale;
  void* q;          // [yrows*4 + h][n][32] FP32 (strict) / BF16 (fast), pre-scaled
  void* k_hi;       // [yrows*4 + h][n][32] tf32 hi (strict) / BF16 (fast)
  void* k_lo;       // strict: tf32 lo of k
  void* v_hi;       // v^T [(yrows*4 + h)*32 + d][ldv], tf32 hi (strict) / BF16 (fast)
  void* v_lo;       // strict: tf32 lo of v^T
  int ldv;          // keys pitch of v^T
  float* bias;      // j-blocked pair bias (bias_index), global rows
  int ldb;
  float* mbias;     // [yrows][ldb] or null
  void* gate;       // [yrows * n][128]: sigmoid(x Wg^T + b_g), fp32 (strict) / bf16 (fast)
  const float* b_g;  // [128] or null
  int* status;
};

// Weight ring depth of the projection (two 32 KB strict stages beside the
// 128 KB A tile and the bias tables); the ring runs across the persistent
// tiles, so the next tile's first weights load during the epilogue.
constexpr int kAttnProjWStages = 2;

template <bool kStrict>
constexpr int attn_proj_smem_bytes() {
  using C = RowCfg<kStrict>;
  return tmem_safe_smem(
      C::A_BYTES + kAttnProjWStages * C::WSTAGE_BYTES + 1024 + 256 + 3 * 4 * 128 * 4, 512);
}

// Persistent, warp-specialised: CTA b takes tiles b, b + gridDim.x, ...
//   LN warps (0-3):       LayerNorm of the tile into A once the previous
//                         tile's MMAs have read it, the 4-head pair bias on
//                         the CUDA cores, the pair / mask bias rows;
//   epilogue warps (4-7): q, k, v^T and gate parts from TMEM to global
//                         memory, each part released as soon as it is read,
//                         so the next tile's MMAs of that part overlap the rest;
//   TMA warp (8):         the weight ring, continuous across tiles;
//   MMA warp (9):         parts q, k, v, gate of each tile (TMEM columns
//                         [0, 512), 128 each).
// Outputs (plain layouts, written by coalesced stores): q / k
// [row*4 + h][j][32] (one thread = one j: 128 contiguous bytes per head),
// v^T [(row*4 + h)*32 + d][key] (a warp's stores to one d are 32
// consecutive keys), gate [row * n + j][128] (one thread = one j).
template <bool kStrict, bool kTrans>
__global__ void __launch_bounds__(320, 1)
    attn_proj_kernel(const __grid_constant__ CUtensorMap w_hi,
                     const __grid_constant__ CUtensorMap w_lo,
                     const __grid_constant__ CUtensorMap zmap, AttnProjArgs p) {
  using C = RowCfg<kStrict>;
  constexpr int WSTAGES = kAttnProjWStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* A = smem;
  uint8_t* W = smem + C::A_BYTES;
  float* bias_tile = reinterpret_cast<float*>(W + WSTAGES * C::WSTAGE_BYTES);  // [4][128]
  float* wb = bias_tile + 4 * 128;                                              // [4][128]
  float* bg = wb + 4 * 128;                                                     // [128] (+pad)
  uint64_t* bars = reinterpret_cast<uint64_t*>(bg + 4 * 128);
  uint64_t* wfull = bars;
  uint64_t* wempty = bars + WSTAGES;
  uint64_t* a_full = bars + 2 * WSTAGES;
  uint64_t* done = a_full + 1;  // [4]: part q, k, v, gate accumulated
  uint64_t* freed = done + 4;   // [4]: part read by the epilogue
  uint64_t* z_full = freed + 4; // strict: raw z rows of the tile in A (TMA)
  uint64_t* drain = z_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = p.n;
  // tile = (y row r, 128-column block): a tile never straddles two rows
  const int njb = (n + 127) / 128;
  const int ntiles = p.yrows * njb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < WSTAGES; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    mbar_init(a_full, 128);
    for (int q = 0; q < 4; ++q) {
      mbar_init(&done[q], 1);
      mbar_init(&freed[q], 128);
    }
    mbar_init(z_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 4 * 128; i += blockDim.x) wb[i] = p.w_bias[i];
  for (int i = threadIdx.x; i < 128; i += blockDim.x) bg[i] = p.b_g ? p.b_g[i] : 0.0f;
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Guard g{p.status, abort_flag};
  const WRing ring{W, wfull, wempty, WSTAGES, C::WSTAGE_BYTES};
  constexpr int NLOADS = 4 * C::NKA;

  if (warp < 4) {
    const float4 lw = reinterpret_cast<const float4*>(p.ln_w)[lane];
    const float4 lb = reinterpret_cast<const float4*>(p.ln_b)[lane];
    float4 wbh[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) wbh[h] = reinterpret_cast<const float4*>(wb + h * 128)[lane];
    const float4* z4 = reinterpret_cast<const float4*>(p.z);
    const int t = warp * 32 + lane;
#pragma unroll 1
    for (int it = 0, tile = blockIdx.x; tile < ntiles; ++it, tile += gridDim.x) {
      const int r = tile / njb, s0 = (tile % njb) * 128;
      if (it > 0 && !mbar_wait(&done[3], (it - 1) & 1, g, 5)) break;
      auto src = [&](int row) -> const float4* {
        const int s = s0 + row;
        if (s >= n) return nullptr;
        return z4 + (kTrans ? ((long long)s * n + r) : ((long long)r * n + s)) * 32;
      };
      // the 4-head pair bias of each row, on the CUDA cores
      auto head_bias = [&](int row, float4 y) {
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float b = warp_sum(y.x * wbh[h].x + y.y * wbh[h].y + y.z * wbh[h].z +
                                   y.w * wbh[h].w);
          if (lane == h) bias_tile[h * 128 + row] = b;
        }
      };
      if constexpr (kStrict) {
        // the tile's raw z rows into the lo half of A by TMA, then
        // LayerNorm in place
        if (threadIdx.x == 0) {
          mbar_arrive_expect_tx(z_full, C::A_SPLIT_BYTES);
#pragma unroll
          for (int a = 0; a < C::NKA; ++a)
            tma_load_3d(A + C::A_SPLIT_BYTES + a * C::ATOM_BYTES, &zmap, z_full, a * C::KATOM,
                        kTrans ? r : s0, kTrans ? s0 : r);
        }
        if (!mbar_wait(z_full, it & 1, g, 7)) break;
        ln_smem_rows_to_a<32>(A, warp * 32, lw, lb, p.eps, head_bias);
      } else {
        ln_rows_to_a<kStrict, 8, true>(A, warp * 32, src, lw, lb, p.eps, head_bias);
      }
      fence_proxy_async_smem();
      mbar_arrive(a_full);
      __syncwarp();  // this warp's rows of bias_tile are complete
      const int s = s0 + t;
      if (s < n) {
#pragma unroll
        for (int h = 0; h < 4; ++h)
          p.bias[bias_index(p.r0 + r, h, s, p.ldb)] = bias_tile[h * 128 + t];
        if (p.mbias) {
          const float m =
              __ldg(p.mask + (kTrans ? ((size_t)s * n + r) : ((size_t)(p.r0 + r) * n + s)));
          p.mbias[(size_t)r * p.ldb + s] = kMaskInf * (m - 1.0f);
        }
      }
      __syncwarp();  // bias_tile is rewritten by the next tile's LayerNorm
    }
  } else if (warp < 8) {
    const int quad = warp & 3;
    const int t = quad * 32 + lane;
    const size_t ldv = (size_t)p.ldv;
#pragma unroll 1
    for (int it = 0, tile = blockIdx.x; tile < ntiles; ++it, tile += gridDim.x) {
      const int r = tile / njb, s0 = (tile % njb) * 128;
      const int j = s0 + t;
      const bool valid = j < n;
      bool ok = true;
#pragma unroll 1
      for (int part = 0; part < 4; ++part) {
        if (!mbar_wait(&done[part], it & 1, g, 3)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // two heads per TMEM round trip; the part is released after the last
#pragma unroll 1
        for (int hp = 0; hp < 2; ++hp) {
          uint32_t vr[2][32];
#pragma unroll
          for (int u = 0; u < 2; ++u)
            tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + part * 128 + (2 * hp + u) * 32,
                      vr[u]);
          tmem_ld_wait();
          if (hp == 1) {
            tc_fence_before();
            mbar_arrive(&freed[part]);  // the next tile's MMAs may reuse these columns
          }
          if (!valid) continue;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const size_t ih = (size_t)r * kHeads + 2 * hp + u;
            if (part < 2) {
              const float sc = part == 0 ? p.q_scale : 1.0f;
              void* dh = part == 0 ? p.q : p.k_hi;
              const size_t row = (ih * n + j) * 32;
              if constexpr (kStrict) {
                float4* oh = reinterpret_cast<float4*>(static_cast<float*>(dh) + row);
                if (part == 0) {
                  // q as FP32: the attention core splits it when staging Q
#pragma unroll
                  for (int e = 0; e < 8; ++e)
                    oh[e] = make_float4(__uint_as_float(vr[u][4 * e]) * sc,
                                        __uint_as_float(vr[u][4 * e + 1]) * sc,
                                        __uint_as_float(vr[u][4 * e + 2]) * sc,
                                        __uint_as_float(vr[u][4 * e + 3]) * sc);
                  continue;
                }
                // k as tf32 hi / lo: the B operand of the core's S MMAs
                float4* ol = reinterpret_cast<float4*>(static_cast<float*>(p.k_lo) + row);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                  float h0, l0, h1, l1, h2, l2, h3, l3;
                  split_tf32(__uint_as_float(vr[u][4 * e]), h0, l0);
                  split_tf32(__uint_as_float(vr[u][4 * e + 1]), h1, l1);
                  split_tf32(__uint_as_float(vr[u][4 * e + 2]), h2, l2);
                  split_tf32(__uint_as_float(vr[u][4 * e + 3]), h3, l3);
                  oh[e] = make_float4(h0, h1, h2, h3);
                  ol[e] = make_float4(l0, l1, l2, l3);
                }
              } else {
                uint4* oh = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(dh) + row);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  uint32_t w4[4];
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    __nv_bfloat162 b2 =
                        __floats2bfloat162_rn(__uint_as_float(vr[u][8 * e + 2 * q]) * sc,
                                              __uint_as_float(vr[u][8 * e + 2 * q + 1]) * sc);
                    w4[q] = *reinterpret_cast<uint32_t*>(&b2);
                  }
                  oh[e] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
              }
            } else if (part == 3) {
              // gate: channels (2 hp + u) * 32 + e of pair (r, j)
              const int c0 = (2 * hp + u) * 32;
              const size_t row = ((size_t)r * n + j) * 128 + c0;
              if constexpr (kStrict) {
                float4* og = reinterpret_cast<float4*>(static_cast<float*>(p.gate) + row);
#pragma unroll
                for (int e = 0; e < 8; ++e)
                  og[e] = make_float4(sigmoidf_(__uint_as_float(vr[u][4 * e]) + bg[c0 + 4 * e]),
                                      sigmoidf_(__uint_as_float(vr[u][4 * e + 1]) +
                                                bg[c0 + 4 * e + 1]),
                                      sigmoidf_(__uint_as_float(vr[u][4 * e + 2]) +
                                                bg[c0 + 4 * e + 2]),
                                      sigmoidf_(__uint_as_float(vr[u][4 * e + 3]) +
                                                bg[c0 + 4 * e + 3]));
              } else {
                uint4* og = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.gate) + row);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  uint32_t w4[4];
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const int c = 8 * e + 2 * q;
                    __nv_bfloat162 b2 = __floats2bfloat162_rn(
                        sigmoidf_(__uint_as_float(vr[u][c]) + bg[c0 + c]),
                        sigmoidf_(__uint_as_float(vr[u][c + 1]) + bg[c0 + c + 1]));
                    w4[q] = *reinterpret_cast<uint32_t*>(&b2);
                  }
                  og[e] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
                }
              }
            } else {
              // v^T: [ih * 32 + d][key j]
#pragma unroll
              for (int d = 0; d < 32; ++d) {
                const size_t idx = (ih * 32 + d) * ldv + j;
                if constexpr (kStrict) {
                  float hh, ll;
                  split_tf32(__uint_as_float(vr[u][d]), hh, ll);
                  static_cast<float*>(p.v_hi)[idx] = hh;
                  static_cast<float*>(p.v_lo)[idx] = ll;
                } else {
                  static_cast<__nv_bfloat16*>(p.v_hi)[idx] =
                      __float2bfloat16_rn(__uint_as_float(vr[u][d]));
                }
              }
            }
          }
        }
      }
      if (!ok) break;
    }
  } else if (warp == 8) {
    if (lane == 0) {
      int seq = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        for (int q = 0; q < NLOADS; ++q, ++seq) {
          const int nc = q / C::NKA, ka = q % C::NKA;
          if (!wring_push<kStrict>(ring, seq, &w_hi, &w_lo, ka * C::KATOM, nc * 128, g)) {
            ok = false;
            break;
          }
        }
      }
      if (g.aborted()) wring_drain(ring, seq, abort_flag);
    }
  } else {
    if (lane == 0) {
      const uint32_t idesc = kStrict ? idesc_tf32(128, 128) : idesc_bf16(128, 128);
      const uint32_t a_hi = smem_u32(A), a_lo = smem_u32(A + C::A_SPLIT_BYTES);
      bool ok = true;
      int seq = 0;
      for (int it = 0, tile = blockIdx.x; tile < ntiles && ok; ++it, tile += gridDim.x) {
        if (!mbar_wait(a_full, it & 1, g, 4)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int nc = 0; nc < 4 && ok; ++nc) {
          if (it > 0 && !mbar_wait(&freed[nc], (it - 1) & 1, g, 6)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int ka = 0; ka < C::NKA; ++ka, ++seq) {
            const uint32_t w = wring_wait(ring, seq, g);
            if (!w) {
              ok = false;
              break;
            }
            mma_k_atom<kStrict>(tmem + nc * 128, a_hi + ka * C::ATOM_BYTES,
                                a_lo + ka * C::ATOM_BYTES, w, w + C::ATOM_BYTES, idesc, ka == 0);
            wring_release(ring, seq);
          }
          if (ok) umma_commit(&done[nc]);
        }
      }
      if (!ok) {
        umma_commit(drain);
        (void)mbar_wait(drain, 0, Guard{nullptr, abort_flag}, 0);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================
// 2. attention core
// ============================================================================
struct AttnCoreArgs {
  int n;
  const float* bias;   // j-blocked pair bias (bias_index)
  const float* mbias;  // [rows][ldb] or null
  int ldb;
  void* o;             // [rows*n][128] fp32 (strict or o_f32) / bf16 (fast)
  int* status;
  int o_f32;           // write fp32 output in fast mode too
  int empty_nan;       // a row whose every logit is -inf: NaN (softmax) or 0 (SDPA)
  const int* kend;     // [rows] keys to visit per row (key_extent_kernel), or null: all n
  const void* gate;    // [rows*n][128] multiplied into o (fp32 strict / bf16 fast), or null
};

// Keys of pair row i that the attention core must visit: 1 + the last key
// whose mask bias is not exactly -1e9 (mask exactly 0), when the row has a
// key with mask bias exactly 0 (mask 1); otherwise (a fully masked row, or
// fractional masks only) every key, n. Exactness of the skip: in such a row
// the running reference max is at least that unmasked key's logit minus 8 in
// log2 units, so each skipped key's logit, about -1e9 below it, gives
// exp2(<= -1e9) = +0 exactly: P = 0, P V adds 0 to O and 0 to the row sum,
// and a tile whose every key is skipped never moves the reference. The
// result is bit-identical to visiting every key. One warp per row.
__global__ void key_extent_kernel(const float* __restrict__ mbias, int ldb, int rows, int n,
                                  int* __restrict__ kend) {
  const int row = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* m = mbias + (size_t)row * ldb;
  int last = -1;
  bool live = false;
  for (int k = lane; k < n; k += 32) {
    const float v = __ldg(m + k);
    if (v != -kMaskInf) last = k;
    if (v == 0.0f) live = true;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
  live = __any_sync(0xffffffffu, live);
  if (lane == 0) kend[row] = live ? last + 1 : n;
}

// Fast-mode shape of the attention core: keys per tile and resident CTAs
// per SM (the strict shape is fixed at 48 keys, two CTAs). Three CTAs need
// 32-key tiles to fit their TMEM share (128 columns) and registers.
#ifndef FPB_ATTN_BKV_FAST
#define FPB_ATTN_BKV_FAST 48
#endif
#ifndef FPB_ATTN_CTAS_FAST
#define FPB_ATTN_CTAS_FAST 2
#endif

template <bool kStrict>
struct AttnCfg {
  static constexpr int BQ = 128;                       // queries per CTA
  static constexpr int BKV = kStrict ? 48 : FPB_ATTN_BKV_FAST;  // keys per tile
  static constexpr int CTAS = kStrict ? 2 : FPB_ATTN_CTAS_FAST;  // resident per SM
  static constexpr int ESZ = kStrict ? 4 : 2;
  static constexpr int NSPLIT = kStrict ? 2 : 1;
  static constexpr int QK_ROW = 32 * ESZ;              // bytes per q/k row (128 / 64)
  static constexpr int Q_BYTES = BQ * QK_ROW;          // FP32 (strict) or BF16 (fast)
  static constexpr int K_BYTES = BKV * QK_ROW;         // per split
  // V^T atoms: 64-byte rows of 16 fp32 keys (strict, 3 per tile) or
  // 128-byte rows of 64 bf16 keys (fast, 1 per tile; 64-byte rows of 32
  // keys for 32-key tiles), 32 rows (d) each
  static constexpr int V_ROW = (kStrict || BKV <= 32) ? 64 : 128;
  static constexpr int V_ATOM_KEYS = V_ROW / ESZ;
  static constexpr int V_ATOMS = (BKV + V_ATOM_KEYS - 1) / V_ATOM_KEYS;
  static constexpr int V_ATOM_BYTES = 32 * V_ROW;
  static constexpr int V_BYTES = V_ATOMS * V_ATOM_BYTES;  // per split
  static constexpr int KV_STAGE = NSPLIT * (K_BYTES + V_BYTES);
  static constexpr int KV_STAGES = kStrict ? 3 : 8;
  static constexpr int QK_STEPS = QK_ROW / 32;         // 32-byte K steps over d
  static constexpr int KSTEP_KEYS = kStrict ? 8 : 16;  // keys per P V K step
  static constexpr int PV_STEPS = BKV / KSTEP_KEYS;
  // TMEM: two S/P buffers of BKV columns (S(t) is read, then P(t)
  // overwrites it: tf32 P_hi, or bf16 pairs), O (32 columns) and the A
  // operands of the S MMAs (Q_hi and Q_lo, 32 columns each; bf16 Q pairs,
  // 16), so every MMA reads only B from shared memory. Strict mode keeps
  // P_lo of the tile in flight in one region of BKV columns shared by both
  // buffers: the softmax writes P_lo(t) only after P V(t-1) has retired.
  static constexpr int BUF_COLS = BKV;
  static constexpr uint32_t kPLO = 2 * BUF_COLS;  // strict only
  static constexpr uint32_t kO = kStrict ? kPLO + BKV : 2 * BUF_COLS;
  static constexpr uint32_t kQ = kO + 32;
  static constexpr uint32_t kQL = kQ + 32;  // strict only
  static constexpr int Q_COLS = kStrict ? 64 : 16;
  static constexpr int TMEM_COLS = CTAS >= 3 ? 128 : 256;
  static_assert(kQ + Q_COLS <= TMEM_COLS, "TMEM budget");
  static_assert(CTAS * TMEM_COLS <= 512, "TMEM per SM");
  static_assert(BKV % KSTEP_KEYS == 0 && BKV % 16 == 0, "key tile shape");
  static_assert(KV_STAGE % 1024 == 0 && (NSPLIT * K_BYTES) % 1024 == 0, "stage alignment");
  static constexpr int THREADS = 192;  // 4 softmax warps, TMA warp, MMA warp
  static constexpr int SMEM =
      tmem_safe_smem(Q_BYTES + KV_STAGES * KV_STAGE + 1024 + 256, TMEM_COLS);
};

template <bool kStrict>
__device__ __forceinline__ uint64_t qk_desc(uint32_t addr) {
  if constexpr (kStrict)
    return umma_desc_sw128(addr);
  else
    return umma_desc_sw64(addr);
}

// One CTA = 128 queries j of one (pair row i, head h), two CTAs per SM (a
// tcgen05.mma is issued every ~50 cycles by one thread whatever its N below
// 128, so two issuing threads per SM double the small-MMA rate).
//   MMA warp:     S(t) = Q K_t^T -> TMEM buffer t%2;
//                 O += P(t) V_t (P(t) read from the same buffer)
//   softmax warps (thread = query row = TMEM lane):
//                 read S(t), add the pair bias (prefetched a tile ahead)
//                 and the mask bias, exponentiate against a running
//                 reference max, write P(t) over S(t).
// O stays in TMEM for the whole key loop. The reference max of a row only
// moves when the tile max exceeds it by more than 8 in log2 units (P <=
// 2^8), and O and the row sum are then rescaled; numerator and denominator
// always use the same reference, so the result is the exact softmax.
// S(t+2) reuses buffer t%2 once P V(t) has retired, so the softmax of
// tile t+1 never waits on the tensor pipe.
template <bool kStrict>
__global__ void __launch_bounds__(192, AttnCfg<kStrict>::CTAS)
    attn_core_kernel(const __grid_constant__ CUtensorMap mq,
                     const __grid_constant__ CUtensorMap mk_hi,
                     const __grid_constant__ CUtensorMap mk_lo,
                     const __grid_constant__ CUtensorMap mv_hi,
                     const __grid_constant__ CUtensorMap mv_lo, AttnCoreArgs p) {
  using C = AttnCfg<kStrict>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* Q = smem;                                   // [split][BQ x QK_ROW]
  uint8_t* KV = Q + C::Q_BYTES;                        // stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(KV + C::KV_STAGES * C::KV_STAGE);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + C::KV_STAGES;
  uint64_t* s_full = kv_empty + C::KV_STAGES;   // [2 buffers]
  uint64_t* p_full = s_full + 2;                // [2 buffers]
  uint64_t* pv_done = p_full + 2;
  uint64_t* q_tmem = pv_done + 1;               // Q (hi) copied into TMEM
  uint64_t* drain = q_tmem + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = p.n;
  const int jt = blockIdx.x, h = blockIdx.y, i = blockIdx.z;
  const int ih = i * kHeads + h;
  // key tiles of this row: the trailing tiles past its key extent hold only
  // keys whose weight is exactly 0 (key_extent_kernel) and are not visited
  const int nt = p.kend ? max(1, (min(__ldg(p.kend + i), n) + C::BKV - 1) / C::BKV)
                        : (n + C::BKV - 1) / C::BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < C::KV_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 128);
    }
    mbar_init(pv_done, 1);
    mbar_init(q_tmem, 128);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Guard g{p.status, abort_flag};

  if (warp == 4) {
    // ------------------------------------------------------------ TMA
    // the gate rows of this CTA's queries are read once the key loop is
    // done: into L2 now, one 128-byte (strict) / 64-byte (fast) row per query
    if (p.gate) {
      for (int r = lane; r < C::BQ && jt * C::BQ + r < n; r += 32)
        prefetch_l2(static_cast<const uint8_t*>(p.gate) +
                        (((size_t)i * n + jt * C::BQ + r) * 128 + h * 32) * C::ESZ,
                    32 * C::ESZ);
    }
    if (lane == 0) {
      // the Q tile is read by this CTA only; keep L2 for the pair bias
      const uint64_t pol_q = policy_evict_first();
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
      tma_load_3d_hint(Q, &mq, q_full, 0, jt * C::BQ, ih, pol_q);
      int issued = 0;
      for (int t = 0; t < nt; ++t) {
        const int s = t % C::KV_STAGES;
        const uint32_t ph = (t / C::KV_STAGES) & 1;
        if (t >= C::KV_STAGES && !mbar_wait(&kv_empty[s], ph ^ 1, g, 21)) break;
        uint8_t* st = KV + s * C::KV_STAGE;
        uint8_t* vst = st + C::NSPLIT * C::K_BYTES;
        mbar_arrive_expect_tx(&kv_full[s], C::KV_STAGE);
        tma_load_3d(st, &mk_hi, &kv_full[s], 0, t * C::BKV, ih);
        if constexpr (kStrict) tma_load_3d(st + C::K_BYTES, &mk_lo, &kv_full[s], 0, t * C::BKV, ih);
#pragma unroll
        for (int a = 0; a < C::V_ATOMS; ++a) {
          const int key = t * C::BKV + a * C::V_ATOM_KEYS;
          tma_load_3d(vst + a * C::V_ATOM_BYTES, &mv_hi, &kv_full[s], key, 0, ih);
          if constexpr (kStrict)
            tma_load_3d(vst + C::V_BYTES + a * C::V_ATOM_BYTES, &mv_lo, &kv_full[s], key, 0, ih);
        }
        ++issued;
      }
      if (g.aborted()) {
        for (int t = (issued > C::KV_STAGES ? issued - C::KV_STAGES : 0); t < issued; ++t)
          (void)mbar_wait(&kv_full[t % C::KV_STAGES], (t / C::KV_STAGES) & 1,
                          Guard{nullptr, abort_flag}, 0);
        (void)mbar_wait(q_full, 0, Guard{nullptr, abort_flag}, 0);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA
    if (lane == 0) {
      const uint32_t id_s = kStrict ? idesc_tf32(128, C::BKV) : idesc_bf16(128, C::BKV);
      const uint32_t id_o = kStrict ? idesc_tf32(128, 32) : idesc_bf16(128, 32);
      auto issue_s = [&](int t) {
        const uint32_t kst = smem_u32(KV + (t % C::KV_STAGES) * C::KV_STAGE);
        const uint32_t sbuf = tmem + (t & 1) * C::BUF_COLS;
#pragma unroll
        for (int kk = 0; kk < C::QK_STEPS; ++kk) {
          const uint32_t off = kk * 32;
          const uint32_t qa = tmem + C::kQ + kk * 8;  // 8 tf32 / 16 bf16 of d per step
          const uint64_t dkh = qk_desc<kStrict>(kst + off);
          const uint32_t acc = kk == 0 ? 0u : 1u;
          if constexpr (kStrict) {
            const uint64_t dkl = qk_desc<kStrict>(kst + C::K_BYTES + off);
            umma_tf32_ts(sbuf, qa, dkh, id_s, acc);                      // Q_hi K_hi
            umma_tf32_ts(sbuf, qa, dkl, id_s, 1u);                       // Q_hi K_lo
            umma_tf32_ts(sbuf, tmem + C::kQL + kk * 8, dkh, id_s, 1u);   // Q_lo K_hi
          } else {
            umma_bf16_ts(sbuf, qa, dkh, id_s, acc);
          }
        }
        umma_commit(&s_full[t & 1]);
      };
      auto issue_pv = [&](int t) {
        const uint32_t vst =
            smem_u32(KV + (t % C::KV_STAGES) * C::KV_STAGE + C::NSPLIT * C::K_BYTES);
        const uint32_t pa = tmem + (t & 1) * C::BUF_COLS;
        const uint32_t d_o = tmem + C::kO;
#pragma unroll
        for (int kk = 0; kk < C::PV_STEPS; ++kk) {
          const uint32_t acc = (t == 0 && kk == 0) ? 0u : 1u;
          // K step kk: V^T atom key / V_ATOM_KEYS, 32-byte offset in its row
          const int key = kk * C::KSTEP_KEYS;
          const uint32_t vo =
              (key / C::V_ATOM_KEYS) * C::V_ATOM_BYTES + (key % C::V_ATOM_KEYS) * C::ESZ;
          if constexpr (kStrict) {
            const uint64_t dvh = umma_desc_sw64(vst + vo);
            const uint64_t dvl = umma_desc_sw64(vst + C::V_BYTES + vo);
            umma_tf32_ts(d_o, pa + kk * 8, dvh, id_o, acc);             // P_hi V_hi
            umma_tf32_ts(d_o, pa + kk * 8, dvl, id_o, 1u);              // P_hi V_lo
            umma_tf32_ts(d_o, tmem + C::kPLO + kk * 8, dvh, id_o, 1u);  // P_lo V_hi
          } else {
            const uint64_t dv =
                C::V_ROW == 64 ? umma_desc_sw64(vst + vo) : umma_desc_sw128(vst + vo);
            umma_bf16_ts(d_o, pa + kk * 8, dv, id_o, acc);
          }
        }
        umma_commit(pv_done);
      };
      // the softmax warps have copied Q (hi) into TMEM (after q_full)
      bool ok = mbar_wait(q_full, 0, g, 22) && mbar_wait(q_tmem, 0, g, 29);
      if (ok) tc_fence_after();
      // S of the first two tiles fill both buffers
      for (int t = 0; t < 2 && t < nt && ok; ++t) {
        if (!mbar_wait(&kv_full[t], 0, g, 24)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_s(t);
      }
      for (int t = 0; t < nt && ok; ++t) {
        if (!mbar_wait(&p_full[t & 1], (t >> 1) & 1, g, 23)) {
          ok = false;
          break;
        }
        tc_fence_after();
        issue_pv(t);
        umma_commit(&kv_empty[t % C::KV_STAGES]);
        if (t + 2 < nt) {
          const int t2 = t + 2;
          // buffer t%2 holds P(t): S(t+2) overwrites it once P V(t) retired
          if (!mbar_wait(&kv_full[t2 % C::KV_STAGES], (t2 / C::KV_STAGES) & 1, g, 24) ||
              !mbar_wait(pv_done, t & 1, g, 25)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_s(t2);
        }
      }
      if (!ok) {
        umma_commit(drain);
        (void)mbar_wait(drain, 0, Guard{nullptr, abort_flag}, 0);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int quad = warp;
    const int t_row = quad * 32 + lane;  // TMEM lane / query row in the tile
    const int j = jt * C::BQ + t_row;
    const bool jvalid = j < n;
    const uint32_t tb = tmem + ((uint32_t)(quad * 32) << 16);
    // this thread's row of the j-blocked bias: key k at brow[(k >> 2) * 128 + (k & 3)]
    const float* brow = p.bias + bias_index(jvalid ? j : 0, h, 0, p.ldb);
    const float* mrow = p.mbias ? p.mbias + (size_t)i * p.ldb : nullptr;
    constexpr float kLog2e = 1.4426950408889634f;
    constexpr float kRescale = 8.0f;  // log2 units: move the reference past P = 2^8
    const uint64_t pol_bias = policy_evict_last();
    // Additive terms of key tile t, loaded in one batch a tile ahead: the
    // pair bias (a different row per thread) plus the mask bias row (the
    // same for every thread, an L1 hit); -inf past n is applied when the
    // tile is consumed. q.k + (bias + mask) equals the reference's
    // (q.k + mask) + bias: unmasked keys add 0, and for masked keys -1e9
    // absorbs any |x| < 32 in FP32 in either order.
    // key pairs (2e, 2e + 1) of a tile live in one float2: the adds,
    // subtractions, scalings and sums run as packed FP32 pair instructions
    // (the same rounding as two scalar operations)
    constexpr int NP = C::BKV / 2;
    auto load_bias = [&](int t, float2 (&cb)[NP]) {
      const int k0 = t * C::BKV;
      if (jvalid && k0 + C::BKV <= n) {
#pragma unroll
        for (int e4 = 0; e4 < C::BKV / 4; ++e4) {
          const float4 b = ldg_f4_hint(brow + ((k0 >> 2) + e4) * 128, pol_bias);
          cb[2 * e4] = make_float2(b.x, b.y);
          cb[2 * e4 + 1] = make_float2(b.z, b.w);
        }
        if (mrow) {
#pragma unroll
          for (int e4 = 0; e4 < C::BKV / 4; ++e4) {
            const float4 m = ldg_f4_hint(mrow + k0 + 4 * e4, pol_bias);
            cb[2 * e4] = __fadd2_rn(cb[2 * e4], make_float2(m.x, m.y));
            cb[2 * e4 + 1] = __fadd2_rn(cb[2 * e4 + 1], make_float2(m.z, m.w));
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < C::BKV; ++e) {
          const int k = k0 + e;
          const float v = (jvalid && k < n) ? brow[(k >> 2) * 128 + (k & 3)] + (mrow ? mrow[k] : 0.f)
                                            : 0.f;
          if (e & 1)
            cb[e >> 1].y = v;
          else
            cb[e >> 1].x = v;
        }
      }
    };
    // reference max in log2 units (mL = fl(m log2e)); every P of the row is
    // exp2(fl(s log2e - mL)) against the current mL, and O and the row sum
    // are rescaled by exp2(mL_old - mL_new) whenever it moves, so numerator
    // and denominator always share one reference
    float mL = -INFINITY, l_run = 0.f;
    float2 cb[NP];
    load_bias(0, cb);
    // this thread's query row of Q (hi and lo) -> TMEM, the A operands of
    // the S MMAs
    bool ok = mbar_wait(q_full, 0, g, 20);
    if (ok) {
      if constexpr (kStrict) {
        // FP32 q row: split here (hi = tf32 truncation, lo = rest)
        uint32_t qh[32], ql[32];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float4 v = *reinterpret_cast<const float4*>(Q + sw128_offset(t_row, e * 16));
          const float f[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float h, l;
            split_tf32(f[u], h, l);
            qh[4 * e + u] = __float_as_uint(h);
            ql[4 * e + u] = __float_as_uint(l);
          }
        }
        tmem_st32(tb + C::kQ, qh);
        tmem_st32(tb + C::kQL, ql);
      } else {
        uint32_t qr[16];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint4 v = *reinterpret_cast<const uint4*>(Q + sw64_offset(t_row, e * 16));
          qr[4 * e] = v.x;
          qr[4 * e + 1] = v.y;
          qr[4 * e + 2] = v.z;
          qr[4 * e + 3] = v.w;
        }
        tmem_st16(tb + C::kQ, qr);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(q_tmem);
    }
    for (int t = 0; t < nt && ok; ++t) {
      const uint32_t buf = tb + (t & 1) * C::BUF_COLS;
      float2 sv[NP];
      if (!mbar_wait(&s_full[t & 1], (t >> 1) & 1, g, 26)) {
        ok = false;
        break;
      }
      tc_fence_after();
      {
        uint32_t r[C::BKV / 16][16];
#pragma unroll
        for (int c = 0; c < C::BKV / 16; ++c) tmem_ld16(buf + c * 16, r[c]);
        tmem_ld_wait();  // one round trip for the whole tile
#pragma unroll
        for (int c = 0; c < C::BKV / 16; ++c)
#pragma unroll
          for (int e = 0; e < 16; e += 2)
            sv[c * 8 + e / 2] = __fadd2_rn(
                make_float2(__uint_as_float(r[c][e]), __uint_as_float(r[c][e + 1])),
                cb[c * 8 + e / 2]);
      }
      if (t * C::BKV + C::BKV > n) {  // -inf past n (last tile only)
#pragma unroll
        for (int e = 0; e < NP; ++e) {
          if (t * C::BKV + 2 * e >= n) sv[e].x = -INFINITY;
          if (t * C::BKV + 2 * e + 1 >= n) sv[e].y = -INFINITY;
        }
      }
      if (t + 1 < nt) load_bias(t + 1, cb);
      // four independent partial maxima (3-input max: two keys per step)
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < NP; ++e) mx4[e & 3] = fmax3f(mx4[e & 3], sv[e].x, sv[e].y);
      const float mx = fmax3f(mx4[0], mx4[1], fmaxf(mx4[2], mx4[3]));
      const float mxL = mx * kLog2e;
      const bool move = mxL > mL + kRescale;  // always on the first finite tile
      const float mL_new = move ? mxL : mL;
      const float alpha = move ? ex2_approx(mL - mL_new) : 1.0f;
      mL = mL_new;
      // while every logit so far is -inf the reference is -inf: exponentiate
      // against 0 instead, so those entries give exp2(-inf) = 0 and not NaN
      const float m_sub = mL == -INFINITY ? 0.0f : mL;
      // P(t) over S(t) (A operand of P V), 16 keys at a time; strict P_lo
      // waits in registers until P V(t-1) has read the shared P_lo region
      float2 ls2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      uint32_t plo[kStrict ? C::BKV : 1];
      // exponent s log2e - mL, one fused multiply-add per key
      const float2 neg_ml = make_float2(-m_sub, -m_sub);
      const float2 l2e = make_float2(kLog2e, kLog2e);
#pragma unroll
      for (int c = 0; c < C::BKV / 16; ++c) {
        float2 pv[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float2 a = __ffma2_rn(sv[c * 8 + e], l2e, neg_ml);
          pv[e] = make_float2(ex2_approx(a.x), ex2_approx(a.y));
          ls2[e & 1] = __fadd2_rn(ls2[e & 1], pv[e]);
        }
        if constexpr (kStrict) {
          // P_hi over S(t); lo = x - hi (exact) kept for the shared region
          uint32_t part[16];
          float2 hi[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            hi[e] = make_float2(__uint_as_float(__float_as_uint(pv[e].x) & 0xFFFFE000u),
                                __uint_as_float(__float_as_uint(pv[e].y) & 0xFFFFE000u));
            part[2 * e] = __float_as_uint(hi[e].x);
            part[2 * e + 1] = __float_as_uint(hi[e].y);
          }
          tmem_st16(buf + c * 16, part);
          const float2 neg1 = make_float2(-1.0f, -1.0f);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float2 lo = __ffma2_rn(hi[e], neg1, pv[e]);  // x - hi, exact
            plo[c * 16 + 2 * e] = __float_as_uint(lo.x);
            plo[c * 16 + 2 * e + 1] = __float_as_uint(lo.y);
          }
        } else {
          // bf16 pairs: 16 keys -> 8 columns
          uint32_t pk[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(pv[e].x, pv[e].y);
            pk[e] = *reinterpret_cast<uint32_t*>(&b2);
          }
          tmem_st8(buf + c * 8, pk);
        }
      }
      l_run = l_run * alpha + ((ls2[0].x + ls2[0].y) + (ls2[1].x + ls2[1].y));
      // Observe every completion of pv_done in order (a parity wait cannot
      // tell phase k from phase k - 2): P V(t-1) was issued when this tile
      // started, so it has normally retired by now. Then a moved reference
      // rescales O (all P V up to t-1) before P V(t) accumulates into it.
      if (t > 0) {
        if (!mbar_wait(pv_done, (t - 1) & 1, g, 27)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      if constexpr (kStrict) {
#pragma unroll
        for (int c = 0; c < C::BKV / 16; ++c) {
          uint32_t part[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) part[e] = plo[c * 16 + e];
          tmem_st16(tb + C::kPLO + c * 16, part);
        }
      }
      if (t > 0 && __any_sync(0xffffffffu, move)) {
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t ov[16];
          tmem_ld16(tb + C::kO + c * 16, ov);
          tmem_ld_wait();
#pragma unroll
          for (int d = 0; d < 16; ++d) ov[d] = __float_as_uint(__uint_as_float(ov[d]) * alpha);
          tmem_st16(tb + C::kO + c * 16, ov);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[t & 1]);
    }
    if (ok && mbar_wait(pv_done, (nt - 1) & 1, g, 28)) {
      tc_fence_after();
      // l_run is 0 only when every logit of the row was -inf
      const bool empty = l_run == 0.0f;
      const float inv = 1.0f / l_run;
      const float fill = p.empty_nan ? __uint_as_float(0x7fc00000u) : 0.0f;
      float o[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t ov[16];
        tmem_ld16(tb + C::kO + c * 16, ov);
        tmem_ld_wait();
#pragma unroll
        for (int d = 0; d < 16; ++d) o[c * 16 + d] = empty ? fill : __uint_as_float(ov[d]) * inv;
      }
      if (jvalid) {
        const size_t orow = (size_t)i * n + j;
        // the attention gate of this (pair, head), when given (the fused
        // operator): o <- sigmoid(x Wg^T + b_g) * o, FP32 (strict) / BF16 (fast)
        const size_t gofs = orow * 128 + h * 32;
        if (kStrict || p.o_f32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.o) + orow * 128 + h * 32);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float4 v = make_float4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
            if constexpr (kStrict) {
              if (p.gate) {
                const float4 gv =
                    __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(p.gate) + gofs) + e);
                v = make_float4(v.x * gv.x, v.y * gv.y, v.z * gv.z, v.w * gv.w);
              }
            }
            dst[e] = v;
          }
        } else {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.o) + orow * 128 +
                                                h * 32);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (p.gate) {
              const uint4 gv = __ldg(reinterpret_cast<const uint4*>(
                                         static_cast<const __nv_bfloat16*>(p.gate) + gofs) + e);
              const uint32_t g4[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&g4[q]);
                o[8 * e + 2 * q] *= __bfloat162float(b2.x);
                o[8 * e + 2 * q + 1] *= __bfloat162float(b2.y);
              }
            }
            uint32_t w4[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              __nv_bfloat162 b2 = __floats2bfloat162_rn(o[8 * e + 2 * q], o[8 * e + 2 * q + 1]);
              w4[q] = *reinterpret_cast<uint32_t*>(&b2);
            }
            dst[e] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Tensor maps and launch of the attention core over nh = rows x 4 (row,
// head) pairs: q [nh][n][32] (FP32 strict, split by the core; BF16 fast),
// k [nh][n][32] and v^T [nh][32][ldv] (tf32 hi / lo strict; BF16 fast, lo
// unused).
int launch_attn_core(const void* q, const void* k_hi, const void* k_lo, const void* v_hi,
                     const void* v_lo, int n, int rows, int ldv, const AttnCoreArgs& ca,
                     bool strict, cudaStream_t stream) {
  const int esz = strict ? 4 : 2;
  const CUtensorMapDataType dt =
      strict ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const CUtensorMapSwizzle qsw = strict ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const uint64_t rowb = 32ull * esz;
  const uint64_t nh = (uint64_t)rows * kHeads;
  const uint32_t bkv = strict ? AttnCfg<true>::BKV : AttnCfg<false>::BKV;
  const uint32_t vkeys = strict ? AttnCfg<true>::V_ATOM_KEYS : AttnCfg<false>::V_ATOM_KEYS;
  const int vrow = strict ? AttnCfg<true>::V_ROW : AttnCfg<false>::V_ROW;
  const CUtensorMapSwizzle vsw = vrow == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap mq, mkh, mkl, mvh, mvl;
  bool ok = make_map_3d(&mq, q, dt, 32, n, nh, rowb, rowb * n, 32, 128, 1, qsw) &&
            make_map_3d(&mkh, k_hi, dt, 32, n, nh, rowb, rowb * n, 32, bkv, 1, qsw) &&
            make_map_3d(&mvh, v_hi, dt, n, 32, nh, (uint64_t)ldv * esz, (uint64_t)ldv * esz * 32,
                        vkeys, 32, 1, vsw);
  if (strict)
    ok = ok && make_map_3d(&mkl, k_lo, dt, 32, n, nh, rowb, rowb * n, 32, bkv, 1, qsw) &&
         make_map_3d(&mvl, v_lo, dt, n, 32, nh, (uint64_t)ldv * esz, (uint64_t)ldv * esz * 32,
                     vkeys, 32, 1, vsw);
  else {
    mkl = mkh;
    mvl = mvh;
  }
  if (!ok) return kErrArg;
  dim3 grid((n + 127) / 128, kHeads, rows);
  if (strict) {
    auto kern = attn_core_kernel<true>;
    if (int smem_st = set_max_smem(kern, AttnCfg<true>::SMEM)) return smem_st;
    FPB_LAUNCH("triattn_core", stream,
               kern<<<grid, AttnCfg<true>::THREADS, AttnCfg<true>::SMEM, stream>>>(
                   mq, mkh, mkl, mvh, mvl, ca));
  } else {
    auto kern = attn_core_kernel<false>;
    if (int smem_st = set_max_smem(kern, AttnCfg<false>::SMEM)) return smem_st;
    FPB_LAUNCH("triattn_core", stream,
               kern<<<grid, AttnCfg<false>::THREADS, AttnCfg<false>::SMEM, stream>>>(
                   mq, mkh, mkl, mvh, mvl, ca));
  }
  return launch_status();
}

// ============================================================================
// 3. output projection + residual
// ============================================================================
struct AttnOutArgs {
  float* z;
  float* delta;  // when non-null: write the update here and leave z unchanged
  int n;
  int rows;      // pair rows of y owned by this call (n unsharded)
  const float* b_o;  // [128] or null
  int* status;
};

template <bool kStrict>
constexpr int attn_out_smem_bytes() {
  using C = RowCfg<kStrict>;
  return tmem_safe_smem(C::A_BYTES + 2 * C::WSTAGE_BYTES + 1024 + 256 + 1024, 256);
}

// Output projection and residual over tiles of 128 pair rows of y (y row r,
// columns s0..), persistent and warp-specialised. The gated attention output
// g * o (the attention core applied the gate) is the A operand as it is:
//   A warps (0-3):        the tile's g * o rows by TMA into A once the
//                         previous tile's MMAs have read it (fast: BF16 rows
//                         straight into the operand layout; strict: FP32 rows
//                         into the lo half, split into tf32 hi / lo in place);
//   epilogue warps (4-7): y = (g * o) W_o^T + b_o from TMEM (two buffers, so
//                         the next tile's MMAs run during this epilogue),
//                         residual added, rows stored to z (or delta);
//   TMA warp (8):         the W_o ring, continuous across tiles;
//   MMA warp (9):         one GEMM per tile into TMEM buffer tile % 2.
// z rows read and written by a tile are its own (row r * n + s, or s * n + r
// transposed), so tiles in flight never touch each other's rows.
template <bool kStrict, bool kTrans>
__global__ void __launch_bounds__(320, 1)
    attn_out_kernel(const __grid_constant__ CUtensorMap w_hi,
                    const __grid_constant__ CUtensorMap w_lo,
                    const __grid_constant__ CUtensorMap omap, AttnOutArgs p) {
  using C = RowCfg<kStrict>;
  constexpr int WSTAGES = 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* A = smem;
  uint8_t* W = smem + C::A_BYTES;
  float* bvec = reinterpret_cast<float*>(W + WSTAGES * C::WSTAGE_BYTES);  // b_o
  uint64_t* bars = reinterpret_cast<uint64_t*>(bvec + 256);
  uint64_t* wfull = bars;
  uint64_t* wempty = bars + WSTAGES;
  uint64_t* o_full = bars + 2 * WSTAGES;  // g * o rows in A (TMA)
  uint64_t* a_full = o_full + 1;          // A ready for the MMAs
  uint64_t* a_free = a_full + 1;          // the tile's MMAs have read A
  uint64_t* y_full = a_free + 1;          // [2] y of the tile in TMEM buffer b
  uint64_t* y_free = y_full + 2;          // [2] buffer b read by the epilogue
  uint64_t* drain = y_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = p.n;
  const int njb = (n + 127) / 128;
  const int ntiles = p.rows * njb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < WSTAGES; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    mbar_init(o_full, 1);
    mbar_init(a_full, 128);
    mbar_init(a_free, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&y_full[b], 1);
      mbar_init(&y_free[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < 128) bvec[threadIdx.x] = p.b_o ? p.b_o[threadIdx.x] : 0.f;
  if (warp == 9) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Guard g{p.status, abort_flag};
  const WRing ring{W, wfull, wempty, WSTAGES, C::WSTAGE_BYTES};

  if (warp < 4) {
    // ---------------------------------------------------------------- A warps
#pragma unroll 1
    for (int it = 0, tile = blockIdx.x; tile < ntiles; ++it, tile += gridDim.x) {
      const int r = tile / njb, s0 = (tile % njb) * 128;
      // A is free once the previous tile's MMAs have read it
      if (it > 0 && !mbar_wait(a_free, (it - 1) & 1, g, 5)) break;
      if (threadIdx.x == 0) {
        // rows s0.. of y row r; rows past n are zero-filled
        mbar_arrive_expect_tx(o_full, C::A_SPLIT_BYTES);
        uint8_t* dst = kStrict ? A + C::A_SPLIT_BYTES : A;
#pragma unroll
        for (int a = 0; a < C::NKA; ++a)
          tma_load_3d(dst + a * C::ATOM_BYTES, &omap, o_full, a * C::KATOM, s0, r);
      }
      if (!mbar_wait(o_full, it & 1, g, 7)) break;
      if constexpr (kStrict) split_smem_rows_to_a<32>(A, warp * 32);
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(a_full);
    }
  } else if (warp < 8) {
    // ---------------------------------------------------------------- epilogue
    const int quad = warp & 3;
    const int t = quad * 32 + lane;
    const bool residual = p.delta == nullptr;
#pragma unroll 1
    for (int it = 0, tile = blockIdx.x; tile < ntiles; ++it, tile += gridDim.x) {
      const int r = tile / njb, s0 = (tile % njb) * 128;
      const int b = it & 1;
      const bool valid = s0 + t < n;
      const long long zrow_idx =
          kTrans ? (long long)(valid ? s0 + t : 0) * n + r : (long long)r * n + (valid ? s0 + t : 0);
      float4* zrow = reinterpret_cast<float4*>(p.z) + zrow_idx * 32;
      float4* drow = residual ? zrow : reinterpret_cast<float4*>(p.delta) + zrow_idx * 32;
      if (valid && residual) prefetch_l2(zrow, 512);  // the residual row, read chunk by chunk
      float4 zc[8];
#pragma unroll
      for (int v4 = 0; v4 < 8; ++v4)
        zc[v4] = (valid && residual) ? zrow[v4] : make_float4(0.f, 0.f, 0.f, 0.f);
      if (!mbar_wait(&y_full[b], (it >> 1) & 1, g, 3)) break;
      tc_fence_after();
      const uint32_t ycol = b * 128;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        float4 zn[8];
#pragma unroll
        for (int v4 = 0; v4 < 8; ++v4)
          zn[v4] = (cc < 3 && valid && residual) ? zrow[(cc + 1) * 8 + v4]
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        uint32_t yr[32];
        tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + ycol + cc * 32, yr);
        tmem_ld_wait();
        if (cc == 3) {
          tc_fence_before();
          mbar_arrive(&y_free[b]);  // the MMAs of tile it + 2 may overwrite this buffer
        }
        if (valid) {
#pragma unroll
          for (int v4 = 0; v4 < 8; ++v4) {
            float4 o = zc[v4];
            const int c = cc * 32 + 4 * v4;
            o.x += __uint_as_float(yr[4 * v4]) + bvec[c];
            o.y += __uint_as_float(yr[4 * v4 + 1]) + bvec[c + 1];
            o.z += __uint_as_float(yr[4 * v4 + 2]) + bvec[c + 2];
            o.w += __uint_as_float(yr[4 * v4 + 3]) + bvec[c + 3];
            drow[cc * 8 + v4] = o;
          }
        }
#pragma unroll
        for (int v4 = 0; v4 < 8; ++v4) zc[v4] = zn[v4];
      }
    }
  } else if (warp == 8) {
    if (lane == 0) {
      int seq = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        for (int ka = 0; ka < C::NKA; ++ka, ++seq) {
          if (!wring_push<kStrict>(ring, seq, &w_hi, &w_lo, ka * C::KATOM, 0, g)) {
            ok = false;
            break;
          }
        }
      }
      if (g.aborted()) wring_drain(ring, seq, abort_flag);
    }
  } else {
    if (lane == 0) {
      const uint32_t idesc = kStrict ? idesc_tf32(128, 128) : idesc_bf16(128, 128);
      const uint32_t a_hi = smem_u32(A), a_lo = smem_u32(A + C::A_SPLIT_BYTES);
      bool ok = true;
      int seq = 0;
      for (int it = 0, tile = blockIdx.x; tile < ntiles && ok; ++it, tile += gridDim.x) {
        const int b = it & 1;
        if (!mbar_wait(a_full, it & 1, g, 4)) {
          ok = false;
          break;
        }
        // buffer b is overwritten once the epilogue has read tile it - 2
        if (it >= 2 && !mbar_wait(&y_free[b], ((it >> 1) - 1) & 1, g, 6)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int ka = 0; ka < C::NKA; ++ka, ++seq) {
          const uint32_t w = wring_wait(ring, seq, g);
          if (!w) {
            ok = false;
            break;
          }
          mma_k_atom<kStrict>(tmem + b * 128, a_hi + ka * C::ATOM_BYTES,
                              a_lo + ka * C::ATOM_BYTES, w, w + C::ATOM_BYTES, idesc, ka == 0);
          wring_release(ring, seq);
        }
        if (!ok) break;
        umma_commit(a_free);
        umma_commit(&y_full[b]);
      }
      if (!ok) {
        umma_commit(drain);
        (void)mbar_wait(drain, 0, Guard{nullptr, abort_flag}, 0);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// ============================================================================
// host
// ============================================================================
// Workspace of one call: packed weights, q/k/v^T, gate, mask bias, gated
// attention output, and (unsharded calls only) the pair bias. `rows` = pair
// rows of y owned by the call (n when unsharded).
template <class Alloc>
struct TriAttnPlan {
  void *wp_hi = nullptr, *wp_lo = nullptr, *wo_hi = nullptr, *wo_lo = nullptr;
  void *q = nullptr, *k_hi = nullptr, *k_lo = nullptr, *v_hi = nullptr, *v_lo = nullptr;
  void *o = nullptr, *gate = nullptr;
  float *bias = nullptr, *mbias = nullptr;
  int ldv = 0, ldb = 0;
  void plan(Alloc& al, int n, int rows, bool strict, bool with_mask, bool own_bias) {
    auto take = [&](size_t c) -> void* {
      return strict ? (void*)al.template take<float>(c) : (void*)al.template take<__nv_bfloat16>(c);
    };
    wp_hi = take(512 * 128);  // [Wq; Wk; Wv; Wg]
    if (strict) wp_lo = take(512 * 128);
    wo_hi = take(128 * 128);
    if (strict) wo_lo = take(128 * 128);
    const size_t qk = (size_t)rows * n * 128;
    // q: FP32 (strict: split by the attention core while staging Q) or
    // BF16; k, v^T: tf32 hi / lo (strict) or BF16
    q = take(qk);
    k_hi = take(qk);
    if (strict) k_lo = take(qk);
    ldv = padded_ld(n, strict ? 4 : 2);
    const size_t vc = (size_t)rows * kHeads * 32 * ldv;
    v_hi = take(vc);
    if (strict) v_lo = take(vc);
    ldb = padded_ld(n, 4);
    if (own_bias) bias = al.template take<float>(bias_elems(n, ldb));
    if (with_mask) {
      mbias = al.template take<float>((size_t)rows * ldb);
      kend = al.template take<int>((size_t)rows);
    }
    o = take((size_t)rows * n * 128);
    gate = take((size_t)rows * n * 128);
  }
  int* kend = nullptr;
};

// phase 1: LN + q/k/v/gate projection of the call's rows, pair bias of
// those rows (written at their global rows of `bias`), mask bias
template <class Plan>
int triattn_proj_run(const Plan& pl, const float* z_loc, const float* mask, int n, int rows,
                     int r0, bool trans, const float* ln_w, const float* ln_b, const float* w_q,
                     const float* w_k, const float* w_v, const float* w_bias, const float* w_g,
                     const float* b_g, float eps, float* bias, bool strict, int* status,
                     cudaStream_t stream) {
  int st;
  if ((st = pack_weights(PackSrc{{w_q, w_k, w_v, w_g}, 4, 128}, pl.wp_hi, pl.wp_lo, strict,
                         stream)))
    return st;
  CUtensorMap mph, mpl;
  if (!make_weight_maps(pl.wp_hi, pl.wp_lo, 512, strict, &mph, &mpl)) return kErrArg;
  // raw z rows of a tile (strict): [128 rows][32 channels] boxes, rows past
  // n zero-filled; transposed: tile rows are rows of z at column r
  CUtensorMap zm{};
  if (strict) {
    const uint64_t rowb = 128ull * 4, pitch = (uint64_t)n * rowb;
    const bool zok = trans ? make_map_3d(&zm, z_loc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 128, rows,
                                         n, rowb, pitch, 32, 1, 128)
                           : make_map_3d(&zm, z_loc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 128, n,
                                         rows, rowb, pitch, 32, 128, 1);
    if (!zok) return kErrArg;
  }
  const int tiles = rows * ((n + 127) / 128);
  const unsigned grid = (unsigned)(tiles < sm_count() ? tiles : sm_count());
  AttnProjArgs pa{z_loc, mask, n, rows, r0, eps, ln_w, ln_b, w_bias,
                  1.0f / sqrtf((float)kHeadDim), pl.q, pl.k_hi, pl.k_lo, pl.v_hi, pl.v_lo,
                  pl.ldv, bias, pl.ldb, pl.mbias, pl.gate, b_g, status};
  const int smem = strict ? attn_proj_smem_bytes<true>() : attn_proj_smem_bytes<false>();
  auto k = strict ? (trans ? attn_proj_kernel<true, true> : attn_proj_kernel<true, false>)
                  : (trans ? attn_proj_kernel<false, true> : attn_proj_kernel<false, false>);
  if (int smem_st = set_max_smem(k, smem)) return smem_st;
  FPB_LAUNCH("triattn_proj", stream, k<<<grid, 320, smem, stream>>>(mph, mpl, zm, pa));
  return launch_status();
}

// phase 2: attention core over the call's rows (keys = all n; the gate is
// applied to o in its epilogue) + output projection and residual (or delta)
// on those rows
template <class Plan>
int triattn_finish_run(const Plan& pl, float* z_loc, float* delta_out, int n, int rows,
                       bool trans, const float* bias, const float* w_o, const float* b_o,
                       bool strict, int* status, cudaStream_t stream) {
  int st;
  if ((st = pack_weights(PackSrc{{w_o, nullptr, nullptr, nullptr}, 1, 128}, pl.wo_hi, pl.wo_lo,
                         strict, stream)))
    return st;
  CUtensorMap moh, mol;
  if (!make_weight_maps(pl.wo_hi, pl.wo_lo, 128, strict, &moh, &mol)) return kErrArg;
  {
    if (pl.kend) {
      FPB_LAUNCH("key_extent", stream,
                 key_extent_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(pl.mbias, pl.ldb, rows, n,
                                                                      pl.kend));
      if ((st = launch_status())) return st;
    }
    AttnCoreArgs ca{n, bias, pl.mbias, pl.ldb, pl.o, status, 0, 0, pl.kend, pl.gate};
    if ((st = launch_attn_core(pl.q, pl.k_hi, pl.k_lo, pl.v_hi, pl.v_lo, n, rows, pl.ldv, ca,
                               strict, stream)))
      return st;
  }
  AttnOutArgs oa{z_loc, delta_out, n, rows, b_o, status};
  // gated attention output, y coordinates [rows][n][128]: boxes of 128 rows
  // x one 128-byte channel atom, rows past n zero-filled
  const int esz = strict ? 4 : 2;
  CUtensorMap om{};
  if (!make_map_3d(&om, pl.o,
                   strict ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 128,
                   n, rows, 128ull * esz, 128ull * esz * n, 128 / esz, 128, 1))
    return kErrArg;
  const int tiles = rows * ((n + 127) / 128);
  const unsigned grid = (unsigned)(tiles < sm_count() ? tiles : sm_count());
  const int smem = strict ? attn_out_smem_bytes<true>() : attn_out_smem_bytes<false>();
  auto k = strict ? (trans ? attn_out_kernel<true, true> : attn_out_kernel<true, false>)
                  : (trans ? attn_out_kernel<false, true> : attn_out_kernel<false, false>);
  if (int smem_st = set_max_smem(k, smem)) return smem_st;
  FPB_LAUNCH("triattn_out", stream, k<<<grid, 320, smem, stream>>>(moh, mol, om, oa));
  return launch_status();
}

}  // namespace fpb

using namespace fpb;

extern "C" size_t fpb_triattn_workspace_size(int n, int c_z, int heads, int head_dim,
                                             int precision, int with_mask) {
  if (n <= 0 || c_z != 128 || heads != kHeads || head_dim != kHeadDim) return 0;
  if (precision != 0 && precision != 1) return 0;
  WsCounter cnt;
  TriAttnPlan<WsCounter> pl;
  pl.plan(cnt, n, n, precision == 0, with_mask != 0, true);
  return cnt.used;
}

extern "C" int fpb_triattn(float* z, float* delta_out, const float* mask, int n, int c_z,
                           int heads, int head_dim, const float* ln_w, const float* ln_b,
                           const float* w_q, const float* w_k, const float* w_v,
                           const float* w_bias, const float* w_g, const float* b_g,
                           const float* w_o, const float* b_o, float eps, int starting,
                           int precision, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream) {
  if (!z || !ln_w || !ln_b || !w_q || !w_k || !w_v || !w_bias || !w_g || !w_o || !workspace)
    return kErrArg;
  if (c_z != 128 || heads != kHeads || head_dim != kHeadDim || n <= 0) return kErrShape;
  if (precision != 0 && precision != 1) return kErrArg;
  if (!aligned16(z) || !aligned16(workspace) || !aligned16(ln_w) || !aligned16(ln_b))
    return kErrAlign;
  if (delta_out && !aligned16(delta_out)) return kErrAlign;
  const bool strict = precision == 0;
  const bool with_mask = mask != nullptr;
  if (workspace_bytes <
      fpb_triattn_workspace_size(n, c_z, heads, head_dim, precision, with_mask ? 1 : 0))
    return kErrWorkspace;
  WsCursor cur(workspace, workspace_bytes);
  TriAttnPlan<WsCursor> pl;
  pl.plan(cur, n, n, strict, with_mask, true);
  if (!cur.ok) return kErrWorkspace;
  int* status = static_cast<int*>(workspace);
  if (reset_status(workspace, stream)) return kErrCuda;
  const bool trans = !starting;
  int st = triattn_proj_run(pl, z, mask, n, n, 0, trans, ln_w, ln_b, w_q, w_k, w_v, w_bias, w_g,
                            b_g, eps, pl.bias, strict, status, stream);
  if (st) return st;
  return triattn_finish_run(pl, z, delta_out, n, n, trans, pl.bias, w_o, b_o, strict, status,
                            stream);
}

// ---------------------------------------------------------------- row-sharded phases
extern "C" size_t fpb_triattn_bias_ld(int n) { return (size_t)padded_ld(n, 4); }

extern "C" size_t fpb_triattn_shard_workspace_size(int n, int rows, int precision,
                                                   int with_mask) {
  if (n <= 0 || rows <= 0 || (precision != 0 && precision != 1)) return 0;
  WsCounter cnt;
  TriAttnPlan<WsCounter> pl;
  pl.plan(cnt, n, rows, precision == 0, with_mask != 0, false);
  return cnt.used;
}

// Starting-node form on rows [r0, r0 + rows) of z (z_loc = those rows).
// Writes this rank's rows of the j-major pair bias `bias_full` ([n][4][ldb],
// ldb = fpb_triattn_bias_ld(n)); the caller all-gathers it before _finish.
extern "C" int fpb_triattn_shard_proj(const float* z_loc, const float* mask, int n, int rows,
                                      int r0, const float* ln_w, const float* ln_b,
                                      const float* w_q, const float* w_k, const float* w_v,
                                      const float* w_bias, const float* w_g, const float* b_g,
                                      float eps, float* bias_full, int precision,
                                      void* workspace, size_t workspace_bytes,
                                      cudaStream_t stream) {
  if (!z_loc || !bias_full || !workspace || !ln_w || !ln_b || !w_q || !w_k || !w_v || !w_bias ||
      !w_g)
    return kErrArg;
  if (precision != 0 && precision != 1) return kErrArg;
  if (n <= 0 || rows <= 0 || r0 < 0 || r0 + rows > n) return kErrShape;
  if (!aligned16(z_loc) || !aligned16(workspace) || !aligned16(ln_w) || !aligned16(ln_b))
    return kErrAlign;
  const bool strict = precision == 0;
  const bool with_mask = mask != nullptr;
  if (workspace_bytes < fpb_triattn_shard_workspace_size(n, rows, precision, with_mask))
    return kErrWorkspace;
  WsCursor cur(workspace, workspace_bytes);
  TriAttnPlan<WsCursor> pl;
  pl.plan(cur, n, rows, strict, with_mask, false);
  if (reset_status(workspace, stream)) return kErrCuda;
  return triattn_proj_run(pl, z_loc, mask, n, rows, r0, false, ln_w, ln_b, w_q, w_k, w_v, w_bias,
                          w_g, b_g, eps, bias_full, strict, static_cast<int*>(workspace), stream);
}

extern "C" int fpb_triattn_shard_finish(float* z_loc, float* delta_out, int n, int rows,
                                        int with_mask, const float* bias_full, const float* w_o,
                                        const float* b_o, int precision, void* workspace,
                                        size_t workspace_bytes, cudaStream_t stream) {
  if (!z_loc || !bias_full || !workspace || !w_o) return kErrArg;
  if (precision != 0 && precision != 1) return kErrArg;
  if (n <= 0 || rows <= 0) return kErrShape;
  if (!aligned16(z_loc) || !aligned16(workspace)) return kErrAlign;
  if (delta_out && !aligned16(delta_out)) return kErrAlign;
  const bool strict = precision == 0;
  if (workspace_bytes < fpb_triattn_shard_workspace_size(n, rows, precision, with_mask))
    return kErrWorkspace;
  WsCursor cur(workspace, workspace_bytes);
  TriAttnPlan<WsCursor> pl;
  pl.plan(cur, n, rows, strict, with_mask != 0, false);
  return triattn_finish_run(pl, z_loc, delta_out, n, rows, false, bias_full, w_o, b_o, strict,
                            static_cast<int*>(workspace), stream);
}

// ============================================================================
// attention core at the reference's q/k/v boundary
// ============================================================================
namespace fpb {

// q or k [B, H, N, 32] (any strides) -> [(b*H + h)*N + j][32]: strict FP32
// (lo == null: q, split by the core) or tf32 hi / lo (k); fast bf16.
template <bool kStrict>
__global__ void pack_qk_kernel(const float* __restrict__ src, long long s0, long long s1,
                               long long s2, long long s3, int batch, int n, void* dst,
                               void* lo) {
  const long long total = (long long)batch * kHeads * n * 32;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(e & 31);
    const long long row = e >> 5;  // (b*H + h)*n + j
    const int j = (int)(row % n);
    const long long bh = row / n;
    const int h = (int)(bh % kHeads);
    const long long b = bh / kHeads;
    const float v = src[b * s0 + h * s1 + j * s2 + d * s3];
    if constexpr (kStrict) {
      if (lo) {
        float vh, vl;
        split_tf32(v, vh, vl);
        static_cast<float*>(dst)[e] = vh;
        static_cast<float*>(lo)[e] = vl;
      } else {
        static_cast<float*>(dst)[e] = v;
      }
    } else {
      static_cast<__nv_bfloat16*>(dst)[e] = __float2bfloat16_rn(v);
    }
  }
}

// v [B, H, N, 32] (any strides) -> v^T [(b*H + h)*32 + d][ldv], 32x32 tiles,
// tf32 hi / lo (strict) or bf16 (fast).
template <bool kStrict>
__global__ void pack_vt_kernel(const float* __restrict__ src, long long s0, long long s1,
                               long long s2, long long s3, int n, int ldv, void* dst, void* lo) {
  __shared__ float tile[32][33];
  const long long bh = blockIdx.y;
  const int k0 = blockIdx.x * 32;
  const long long b = bh / kHeads;
  const int h = (int)(bh % kHeads);
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    const int k = k0 + y;
    tile[y][threadIdx.x] = k < n ? src[b * s0 + h * s1 + k * s2 + threadIdx.x * s3] : 0.f;
  }
  __syncthreads();
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {  // y = d
    const int k = k0 + threadIdx.x;
    if (k < n) {
      const size_t idx = ((size_t)bh * 32 + y) * ldv + k;
      const float v = tile[threadIdx.x][y];
      if constexpr (kStrict) {
        float vh, vl;
        split_tf32(v, vh, vl);
        static_cast<float*>(dst)[idx] = vh;
        static_cast<float*>(lo)[idx] = vl;
      } else {
        static_cast<__nv_bfloat16*>(dst)[idx] = __float2bfloat16_rn(v);
      }
    }
  }
}

// triangle bias [1, H, N, N] -> j-blocked (bias_index); mask bias [B, 1, 1, N] -> [b][ldb]
__global__ void pack_bias_kernel(const float* __restrict__ tb, long long t1, long long t2,
                                 long long t3, const float* __restrict__ mb, long long m0,
                                 long long m3, int batch, int n, int ldb, float* bias,
                                 float* mbias) {
  const long long nb = (long long)kHeads * n * n;
  const long long nm = mb ? (long long)batch * n : 0;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < nb + nm;
       e += (long long)gridDim.x * blockDim.x) {
    if (e < nb) {
      const int k = (int)(e % n);
      const long long hj = e / n;
      const int j = (int)(hj % n);
      const int h = (int)(hj / n);
      bias[bias_index(j, h, k, ldb)] = tb[h * t1 + j * t2 + k * t3];
    } else {
      const long long f = e - nb;
      const int k = (int)(f % n);
      const long long b = f / n;
      mbias[(size_t)b * ldb + k] = mb[b * m0 + k * m3];
    }
  }
}

template <class Alloc>
struct CorePlan {
  void *q = nullptr, *k_hi = nullptr, *k_lo = nullptr, *v_hi = nullptr, *v_lo = nullptr;
  float *bias = nullptr, *mbias = nullptr;
  int ldv = 0, ldb = 0;
  void plan(Alloc& al, int batch, int n, bool strict, bool with_mask) {
    auto take = [&](size_t c) -> void* {
      return strict ? (void*)al.template take<float>(c) : (void*)al.template take<__nv_bfloat16>(c);
    };
    const size_t qk = (size_t)batch * kHeads * n * 32;
    q = take(qk);
    k_hi = take(qk);
    if (strict) k_lo = take(qk);
    ldv = padded_ld(n, strict ? 4 : 2);
    const size_t vc = (size_t)batch * kHeads * 32 * ldv;
    v_hi = take(vc);
    if (strict) v_lo = take(vc);
    ldb = padded_ld(n, 4);
    bias = al.template take<float>(bias_elems(n, ldb));
    if (with_mask) mbias = al.template take<float>((size_t)batch * ldb);
  }
};

}  // namespace fpb

extern "C" size_t fpb_attention_core_workspace_size(int batch, int n, int heads, int head_dim,
                                                    int precision, int with_mask) {
  if (batch <= 0 || n <= 0 || heads != kHeads || head_dim != kHeadDim) return 0;
  if (precision != 0 && precision != 1) return 0;
  WsCounter cnt;
  CorePlan<WsCounter> pl;
  pl.plan(cnt, batch, n, precision == 0, with_mask != 0);
  return cnt.used;
}

extern "C" int fpb_attention_core_ex(const float* q, const long long* q_strides,
                                     const float* k, const long long* k_strides, const float* v,
                                     const long long* v_strides, int batch, int n, int heads,
                                     int head_dim, const float* tri_bias,
                                     const long long* tri_bias_strides, const float* mask_bias,
                                     const long long* mask_bias_strides, float* out,
                                     int precision, int empty_rows_nan, void* workspace,
                                     size_t workspace_bytes, cudaStream_t stream) {
  if (empty_rows_nan != 0 && empty_rows_nan != 1) return kErrArg;
  if (!q || !k || !v || !q_strides || !k_strides || !v_strides || !tri_bias ||
      !tri_bias_strides || !out || !workspace || (mask_bias && !mask_bias_strides))
    return kErrArg;
  if (heads != kHeads || head_dim != kHeadDim || batch <= 0 || n <= 0) return kErrShape;
  if (precision != 0 && precision != 1) return kErrArg;
  if (!aligned16(out) || !aligned16(workspace)) return kErrAlign;
  const bool strict = precision == 0;
  const bool with_mask = mask_bias != nullptr;
  if (workspace_bytes <
      fpb_attention_core_workspace_size(batch, n, heads, head_dim, precision, with_mask))
    return kErrWorkspace;
  WsCursor cur(workspace, workspace_bytes);
  CorePlan<WsCursor> pl;
  pl.plan(cur, batch, n, strict, with_mask);
  if (!cur.ok) return kErrWorkspace;
  if (reset_status(workspace, stream)) return kErrCuda;
  int st;
  const long long* qs = q_strides;
  const long long* ks = k_strides;
  const long long* vs = v_strides;
  if (strict) {
    FPB_LAUNCH("pack_qkv", stream,
               pack_qk_kernel<true><<<1184, 256, 0, stream>>>(q, qs[0], qs[1], qs[2], qs[3], batch,
                                                              n, pl.q, nullptr));
    FPB_LAUNCH("pack_qkv", stream,
               pack_qk_kernel<true><<<1184, 256, 0, stream>>>(k, ks[0], ks[1], ks[2], ks[3], batch,
                                                              n, pl.k_hi, pl.k_lo));
    FPB_LAUNCH("pack_qkv", stream,
               pack_vt_kernel<true><<<dim3((n + 31) / 32, batch * kHeads), dim3(32, 8), 0,
                                      stream>>>(v, vs[0], vs[1], vs[2], vs[3], n, pl.ldv, pl.v_hi,
                                                pl.v_lo));
  } else {
    FPB_LAUNCH("pack_qkv", stream,
               pack_qk_kernel<false><<<1184, 256, 0, stream>>>(q, qs[0], qs[1], qs[2], qs[3],
                                                               batch, n, pl.q, nullptr));
    FPB_LAUNCH("pack_qkv", stream,
               pack_qk_kernel<false><<<1184, 256, 0, stream>>>(k, ks[0], ks[1], ks[2], ks[3],
                                                               batch, n, pl.k_hi, nullptr));
    FPB_LAUNCH("pack_qkv", stream,
               pack_vt_kernel<false><<<dim3((n + 31) / 32, batch * kHeads), dim3(32, 8), 0,
                                       stream>>>(v, vs[0], vs[1], vs[2], vs[3], n, pl.ldv, pl.v_hi,
                                                 nullptr));
  }
  const long long* tb = tri_bias_strides;
  const long long* mbs = mask_bias_strides;
  FPB_LAUNCH("pack_qkv", stream,
             pack_bias_kernel<<<1184, 256, 0, stream>>>(tri_bias, tb[1], tb[2], tb[3], mask_bias,
                                                        with_mask ? mbs[0] : 0,
                                                        with_mask ? mbs[3] : 0, batch, n, pl.ldb,
                                                        pl.bias, pl.mbias));
  if ((st = launch_status())) return st;
  // this boundary returns FP32 [B, N, H, D] in both precision modes
  AttnCoreArgs ca{n, pl.bias, pl.mbias, pl.ldb, out, static_cast<int*>(workspace), 1,
                  empty_rows_nan};
  return launch_attn_core(pl.q, pl.k_hi, pl.k_lo, pl.v_hi, pl.v_lo, n, batch, pl.ldv, ca, strict,
                          stream);
}

extern "C" int fpb_attention_core(const float* q, const long long* q_strides, const float* k,
                                  const long long* k_strides, const float* v,
                                  const long long* v_strides, int batch, int n, int heads,
                                  int head_dim, const float* tri_bias,
                                  const long long* tri_bias_strides, const float* mask_bias,
                                  const long long* mask_bias_strides, float* out, int precision,
                                  void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return fpb_attention_core_ex(q, q_strides, k, k_strides, v, v_strides, batch, n, heads,
                               head_dim, tri_bias, tri_bias_strides, mask_bias, mask_bias_strides,
                               out, precision, 0, workspace, workspace_bytes, stream);
}
