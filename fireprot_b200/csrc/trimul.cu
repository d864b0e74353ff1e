// Triangle multiplicative update (outgoing / incoming), fused on sm_100a.
//
// Reference operator: Protenix TriangleMultiplicativeUpdate as dispatched by
// python/fireprot/backends/amd/triangle_multiplication.py:389-430 (math at
// :162-193, contraction directions at lt_bmm.py:85):
//   zn = LN_in(z); a = mask * sigmoid(zn Wag^T) * (zn Wap^T); b likewise
//   outgoing x_ij = sum_k a_ik b_jk ; incoming x_ij = sum_k a_ki b_kj
//   z <- [z +] sigmoid(zn Wg^T) * (LN_out(x) Wz^T)
//
// Three launches per call:
//  1. proj:     LN_in + [Wap;Wag;Wbp;Wbg] GEMM (128 x 512 per tile, TMEM
//               512 columns) + gate/mask epilogue writing a, b channel-first
//               [c][i][k] (3xTF32 hi/lo split in strict mode). The incoming
//               direction reads z transposed (pair (i,k) <- z[k][i]) so that
//               the contraction is always "A B^T".
//  2. contract: batched tcgen05 N^3 contraction (contract.cu) -> x [c][i][j].
//  3. out:      LN_in(z) Wg^T and LN_out(x) Wz^T (two 128x128 GEMMs sharing
//               one A buffer) + sigmoid gate + residual, written in place.
#include "kernels.h"
#include "rowgemm.cuh"

namespace fpb {

// y coordinates: y is a yrows x ycols grid of pair rows; pair (r, s) of y
// is z_loc[r][s] (outgoing) or z_loc[s][r] (incoming, z read transposed),
// where z_loc is the [rows][zcols] block of z this call owns and r0 its first
// global row (for the [N][N] mask).
struct TriMulProjArgs {
  const float* z;
  const float* mask;  // nullable, [N][N] global
  int yrows, ycols, zcols, r0;
  float eps;
  const float* ln_w;
  const float* ln_b;
  void* a_hi;
  void* a_lo;
  void* b_hi;
  void* b_lo;
  int ld;
  size_t cs;
  int* status;
  int b_plain;  // strict: write b unsplit (FP32) into the b_hi planes
  int ntiles;   // yrows x ceil(ycols / 128) tiles, walked by a persistent grid
  int a_plain;  // strict: write a unsplit (FP32) into the a_hi planes
  // Owner scatter (owners > 0; a and b unsplit): channel c goes to the
  // receive buffer of rank c / gch, plane (rank * gch + c % gch) of its
  // [owners][gch][plane_rows][ld] layout (peer addresses for other ranks).
  int owners;
  int gch;
  int rank;
  void* a_out[16];
  void* b_out[16];
};

// Weight ring depth of the projection kernel: three 32 KB strict stages
// plus the 128 KB A tile fit in 227 KB; the ring runs across tiles, so the
// first weights of the next tile load during the current epilogue.
constexpr int kProjWStages = 3;

template <bool kStrict>
constexpr int proj_smem_bytes() {
  using C = RowCfg<kStrict>;
  return tmem_safe_smem(C::A_BYTES + kProjWStages * C::WSTAGE_BYTES + 1024 + 256, 512);
}

template <bool kStrict, bool kTrans>
__global__ void __launch_bounds__(320, 1)
    trimul_proj_kernel(const __grid_constant__ CUtensorMap w_hi,
                       const __grid_constant__ CUtensorMap w_lo,
                       const __grid_constant__ CUtensorMap zmap, TriMulProjArgs p) {
  using C = RowCfg<kStrict>;
  constexpr int WSTAGES = kProjWStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* A = smem;
  uint8_t* W = smem + C::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(W + WSTAGES * C::WSTAGE_BYTES);
  uint64_t* wfull = bars;
  uint64_t* wempty = bars + WSTAGES;
  uint64_t* a_full = bars + 2 * WSTAGES;  // A of the tile written (LN warps)
  uint64_t* done_a = a_full + 1;          // accumulators of part a ready (MMA)
  uint64_t* done_b = done_a + 1;          // part b ready; every MMA of the tile read A
  uint64_t* free_a = done_b + 1;          // part a accumulators read (epilogue warps)
  uint64_t* free_b = free_a + 1;          // part b accumulators read
  uint64_t* z_full = free_b + 1;          // strict: raw z rows of the tile in A (TMA)
  uint64_t* drain = z_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // tile = (y row r, 128-column block jb): a tile never straddles two y rows.
  // The grid is persistent: CTA b takes tiles b, b + gridDim.x, ...
  const int njb = (p.ycols + 127) / 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < WSTAGES; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    mbar_init(a_full, 128);
    mbar_init(done_a, 1);
    mbar_init(done_b, 1);
    mbar_init(free_a, 128);
    mbar_init(free_b, 128);
    mbar_init(z_full, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
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
  constexpr int NLOADS = 4 * C::NKA;  // 4 chunks of 128 outputs x K atoms

  if (warp < 4) {
    // ---- LayerNorm warps: 32 rows each into A, once the MMAs of the
    // previous tile have read it
    const float4 lw = reinterpret_cast<const float4*>(p.ln_w)[lane];
    const float4 lb = reinterpret_cast<const float4*>(p.ln_b)[lane];
    const float4* z4 = reinterpret_cast<const float4*>(p.z);
#pragma unroll 1
    for (int it = 0, tile = blockIdx.x; tile < p.ntiles; ++it, tile += gridDim.x) {
      const int r = tile / njb, s0 = (tile % njb) * 128;
      if (it > 0 && !mbar_wait(done_b, (it - 1) & 1, g, 5)) break;
      if constexpr (kStrict) {
        // the tile's raw z rows into the lo half of A by TMA (one 64 KB
        // transfer instead of per-warp row loads), then LayerNorm in place
        if (threadIdx.x == 0) {
          mbar_arrive_expect_tx(z_full, C::A_SPLIT_BYTES);
#pragma unroll
          for (int a = 0; a < C::NKA; ++a)
            tma_load_3d(A + C::A_SPLIT_BYTES + a * C::ATOM_BYTES, &zmap, z_full, a * C::KATOM,
                        kTrans ? r : s0, kTrans ? s0 : r);
        }
        if (!mbar_wait(z_full, it & 1, g, 7)) break;
        ln_smem_rows_to_a<32>(A, warp * 32, lw, lb, p.eps, NoRowHook{});
      } else {
        auto src = [&](int row) -> const float4* {
          const int sc = s0 + row;
          if (sc >= p.ycols) return nullptr;
          return z4 +
                 (kTrans ? ((long long)sc * p.zcols + r) : ((long long)r * p.zcols + sc)) * 32;
        };
        ln_rows_to_a<kStrict, 16, true>(A, warp * 32, src, lw, lb, p.eps, NoRowHook{});
      }
      fence_proxy_async_smem();
      mbar_arrive(a_full);
    }
  } else if (warp < 8) {
    // ---- epilogue warps: thread t owns tile row t (TMEM lane t) =
    // column s0 + t of every output plane; a warp's stores to one channel
    // are 32 consecutive columns (128 coalesced bytes in strict mode)
    const int quad = warp & 3;
    const int t = quad * 32 + lane;
#pragma unroll 1
    for (int it = 0, tile = blockIdx.x; tile < p.ntiles; ++it, tile += gridDim.x) {
      const int r = tile / njb, s0 = (tile % njb) * 128;
      const int s = s0 + t;
      const bool valid = s < p.ycols;
      float m = 1.f;
      if (p.mask && valid)
        m = __ldg(p.mask + (kTrans ? ((size_t)(p.r0 + s) * p.zcols + r)
                                   : ((size_t)(p.r0 + r) * p.zcols + s)));
      const size_t pos = (size_t)r * p.ld + (valid ? s : 0);
      bool ok = true;
#pragma unroll 1
      for (int part = 0; part < 2 && ok; ++part) {
        if (!mbar_wait(part ? done_b : done_a, it & 1, g, 3)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool plain = kStrict && (part ? p.b_plain : p.a_plain);
        void* ph = part ? p.b_hi : p.a_hi;
        void* pl = part ? p.b_lo : p.a_lo;
#pragma unroll 1
        for (int cc = 0; cc < 4; ++cc) {
          uint32_t pr[32], gr[32];
          const uint32_t base = tmem + ((uint32_t)(quad * 32) << 16) + part * 256 + cc * 32;
          tmem_ld32(base, pr);
          tmem_ld32(base + 128, gr);
          tmem_ld_wait();
          if (cc == 3) {
            // the last TMEM read of this part: the next tile's MMAs may
            // overwrite these columns while the values below are stored
            tc_fence_before();
            mbar_arrive(part ? free_b : free_a);
          }
          if (!valid) continue;
          if (p.owners) {
            // straight into the owners' receive buffers (one channel group
            // per rank): the exchange rides on the epilogue's stores
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              const float v = sigmoidf_(__uint_as_float(gr[e])) * __uint_as_float(pr[e]) * m;
              const int c = cc * 32 + e, grp = c / p.gch;
              const size_t idx = (size_t)(p.rank * p.gch + c - grp * p.gch) * p.cs + pos;
              void* dst = part ? p.b_out[grp] : p.a_out[grp];
              if constexpr (kStrict)
                static_cast<float*>(dst)[idx] = v;
              else
                static_cast<__nv_bfloat16*>(dst)[idx] = __float2bfloat16_rn(v);
            }
            continue;
          }
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float v = sigmoidf_(__uint_as_float(gr[e])) * __uint_as_float(pr[e]) * m;
            const size_t idx = (size_t)(cc * 32 + e) * p.cs + pos;
            if constexpr (kStrict) {
              float h, l;
              split_tf32(v, h, l);
              static_cast<float*>(ph)[idx] = plain ? v : h;
              if (!plain) static_cast<float*>(pl)[idx] = l;
            } else {
              static_cast<__nv_bfloat16*>(ph)[idx] = __float2bfloat16_rn(v);
            }
          }
        }
      }
      if (!ok) break;
    }
  } else if (warp == 8) {
    if (lane == 0) {
      // the same weight sequence for every tile; the ring runs across tiles
      int seq = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < p.ntiles && ok; tile += gridDim.x) {
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
      for (int it = 0, tile = blockIdx.x; tile < p.ntiles && ok; ++it, tile += gridDim.x) {
        if (!mbar_wait(a_full, it & 1, g, 4)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // part a (chunks 0, 1: a_p, a_g), then part b (chunks 2, 3), each
        // once the epilogue has read that part of the previous tile
        for (int part = 0; part < 2 && ok; ++part) {
          if (it > 0 && !mbar_wait(part ? free_b : free_a, (it - 1) & 1, g, 6)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int q = part * 2 * C::NKA; q < (part + 1) * 2 * C::NKA; ++q, ++seq) {
            const int nc = q / C::NKA, ka = q % C::NKA;
            const uint32_t w = wring_wait(ring, seq, g);
            if (!w) {
              ok = false;
              break;
            }
            mma_k_atom<kStrict>(tmem + nc * 128, a_hi + ka * C::ATOM_BYTES,
                                a_lo + ka * C::ATOM_BYTES, w, w + C::ATOM_BYTES, idesc, ka == 0);
            wring_release(ring, seq);
          }
          if (ok) umma_commit(part ? done_b : done_a);
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

// ----------------------------------------------------------------------------
struct TriMulOutArgs {
  float* z;
  int n;
  float eps_in, eps_out;
  const float* ln_in_w;
  const float* ln_in_b;
  const float* ln_out_w;
  const float* ln_out_b;
  const void* x;  // blocked [n][njb][128 c][128 j] fp32 (strict) or bf16 (fast)
  int njb;
  int add;
  int* status;
  int ntiles;  // rows x njb tiles, walked by a persistent grid
};

// Element (channel c, tile row t) of a blocked x tile.
template <bool kStrict>
__device__ __forceinline__ float x_at(const void* tile, int c, int t) {
  if constexpr (kStrict)
    return __ldg(static_cast<const float*>(tile) + c * 128 + t);
  else
    return __bfloat162float(static_cast<const __nv_bfloat16*>(tile)[c * 128 + t]);
}

template <bool kStrict>
constexpr int out_smem_bytes() {
  using C = RowCfg<kStrict>;
  return tmem_safe_smem(C::A_BYTES + 2 * C::WSTAGE_BYTES + 1024 + 256 + 1024, 512);
}

// Persistent: one CTA per SM walks tiles blockIdx.x, +gridDim.x, ... Per
// tile, GEMM 1 (gate G = LN_in(z) Wg^T) and GEMM 2 (Y = LN_out(x) Wz^T)
// share the A tile and write one of two TMEM buffers (256 columns each), so
// the epilogue of the previous tile runs while GEMM 1 of this one executes,
// the x row loads overlap GEMM 1 and the next tile's z rows are prefetched
// into registers during GEMM 2. The weight ring runs on across tiles.
// Row warps, per tile i:
//   wait GEMM 2(i-1) -> LN_in(z_i) into A -> epilogue(i-1) -> load x_i ->
//   wait GEMM 1(i) -> LN_out(x_i) into A -> prefetch z_{i+1}
template <bool kStrict>
__global__ void __launch_bounds__(192, 1)
    trimul_out_kernel(const __grid_constant__ CUtensorMap w_hi,
                      const __grid_constant__ CUtensorMap w_lo, TriMulOutArgs p) {
  using C = RowCfg<kStrict>;
  constexpr int WSTAGES = 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* A = smem;
  uint8_t* W = smem + C::A_BYTES;
  float* lnp = reinterpret_cast<float*>(W + WSTAGES * C::WSTAGE_BYTES);  // 256 floats
  uint64_t* bars = reinterpret_cast<uint64_t*>(lnp + 256);
  uint64_t* wfull = bars;
  uint64_t* wempty = bars + WSTAGES;
  uint64_t* a_full = bars + 2 * WSTAGES;  // LN_in / LN_out of a tile written to A
  uint64_t* gdone = a_full + 1;           // GEMM 1 / GEMM 2 of a tile retired
  uint64_t* tfree = gdone + 1;            // [2] epilogue done reading a TMEM buffer
  uint64_t* drain = tfree + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = p.n;
  const int ntiles = p.ntiles;
  const int nmine = blockIdx.x < ntiles ? (ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < WSTAGES; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    mbar_init(a_full, 128);
    mbar_init(gdone, 1);
    mbar_init(&tfree[0], 128);
    mbar_init(&tfree[1], 128);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < 128) {
    lnp[threadIdx.x] = p.ln_out_w[threadIdx.x];
    lnp[128 + threadIdx.x] = p.ln_out_b[threadIdx.x];
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Guard g{p.status, abort_flag};
  const WRing ring{W, wfull, wempty, WSTAGES, C::WSTAGE_BYTES};
  constexpr int NLOADS = 2 * C::NKA;  // per tile: GEMM 1 then GEMM 2, K atoms each

  if (warp < 4) {
    const int t = warp * 32 + lane;  // tile row (TMEM lane)
    const float4 lw = reinterpret_cast<const float4*>(p.ln_in_w)[lane];
    const float4 lb = reinterpret_cast<const float4*>(p.ln_in_b)[lane];
    const float4* z4 = reinterpret_cast<const float4*>(p.z);
    // tile -> (pair row i, 128-column block jb); rows never straddle i
    auto tile_p0 = [&](int tile) { return (long long)(tile / p.njb) * n + (tile % p.njb) * 128; };
    auto tile_rows = [&](int tile) { return min(128, n - (tile % p.njb) * 128); };
    // z rows of this warp's 32 tile rows, lane-cooperative (lane = 4 channels)
    float4 zr[32];
    auto load_z = [&](int tile) {
      const long long p0 = tile_p0(tile);
      const int valid = tile_rows(tile);
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int row = warp * 32 + u;
        zr[u] = row < valid ? z4[(p0 + row) * 32 + lane] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    };
    auto epilogue = [&](int tile, int b) {
      // delta = sigmoid(G) * Y, z <- [z +] delta; thread t owns row t
      const long long p0 = tile_p0(tile);
      const bool valid = t < tile_rows(tile);
      const uint32_t tb = tmem + b * 256;
      float4* zrow = reinterpret_cast<float4*>(p.z) + (p0 + (valid ? t : 0)) * 32;
      float4 zc[8];
#pragma unroll
      for (int v4 = 0; v4 < 8; ++v4)
        zc[v4] = (valid && p.add) ? zrow[v4] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        float4 zn[8];
#pragma unroll
        for (int v4 = 0; v4 < 8; ++v4)
          zn[v4] = (cc < 3 && valid && p.add) ? zrow[(cc + 1) * 8 + v4]
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
        float gv[32], yv[32];
        tmem_row32(tb, warp, cc * 32, gv);
        tmem_row32(tb, warp, 128 + cc * 32, yv);
        if (valid) {
#pragma unroll
          for (int v4 = 0; v4 < 8; ++v4) {
            float4 o = zc[v4];
            o.x += sigmoidf_(gv[4 * v4]) * yv[4 * v4];
            o.y += sigmoidf_(gv[4 * v4 + 1]) * yv[4 * v4 + 1];
            o.z += sigmoidf_(gv[4 * v4 + 2]) * yv[4 * v4 + 2];
            o.w += sigmoidf_(gv[4 * v4 + 3]) * yv[4 * v4 + 3];
            zrow[cc * 8 + v4] = o;
          }
        }
#pragma unroll
        for (int v4 = 0; v4 < 8; ++v4) zc[v4] = zn[v4];
      }
    };
    bool ok = true;
    if (nmine > 0) load_z(blockIdx.x);
    for (int it = 0; it < nmine && ok; ++it) {
      const int tile = blockIdx.x + it * gridDim.x;
      // A is free once GEMM 2 of the previous tile retired
      if (it > 0) {
        if (!mbar_wait(gdone, 1, g, 5)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      // ---- A1 = LN_in(z) from the prefetched rows
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const float4 y = ln_row_warp(zr[u], lw, lb, p.eps_in);
        a_store4<kStrict>(A, warp * 32 + u, lane * 4, y.x, y.y, y.z, y.w);
      }
      fence_proxy_async_smem();
      mbar_arrive(a_full);
      // ---- epilogue of the previous tile (overlaps GEMM 1 of this one)
      if (it > 0) {
        const int pb = (it - 1) & 1;
        epilogue(tile - (int)gridDim.x, pb);
        tc_fence_before();
        mbar_arrive(&tfree[pb]);
      }
      // ---- A2 = LN_out(x): thread t loads its row's 128 channels in one batch
      {
        const size_t tile_elems = (size_t)tile * 128 * 128;
        const void* xt = kStrict ? (const void*)(static_cast<const float*>(p.x) + tile_elems)
                                 : (const void*)(static_cast<const __nv_bfloat16*>(p.x) + tile_elems);
        float xv[128];
#pragma unroll
        for (int c = 0; c < 128; ++c) xv[c] = x_at<kStrict>(xt, c, t);
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 128; ++c) s4[c & 3] += xv[c];
        const float mean = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * (1.0f / 128.0f);
        float q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < 128; ++c) {
          const float d = xv[c] - mean;
          q4[c & 3] += d * d;
        }
        const float var = ((q4[0] + q4[1]) + (q4[2] + q4[3])) * (1.0f / 128.0f);
        const float rs = rsqrtf(var + p.eps_out);
        // GEMM 1 must have finished reading A before it is reused
        if (!mbar_wait(gdone, 0, g, 6)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 128; c += 4)
          a_store4<kStrict>(A, t, c, (xv[c] - mean) * rs * lnp[c] + lnp[128 + c],
                            (xv[c + 1] - mean) * rs * lnp[c + 1] + lnp[129 + c],
                            (xv[c + 2] - mean) * rs * lnp[c + 2] + lnp[130 + c],
                            (xv[c + 3] - mean) * rs * lnp[c + 3] + lnp[131 + c]);
        fence_proxy_async_smem();
        mbar_arrive(a_full);
      }
      // ---- next tile's z rows (overlap GEMM 2); the last iteration reloads
      // its own tile so that zr is always redefined here (never live across
      // the epilogue and LN_out)
      load_z(it + 1 < nmine ? tile + (int)gridDim.x : tile);
    }
    // ---- last tile's epilogue
    if (ok && nmine > 0 && mbar_wait(gdone, 1, g, 7)) {
      tc_fence_after();
      epilogue(blockIdx.x + (nmine - 1) * gridDim.x, (nmine - 1) & 1);
    }
  } else if (warp == 4) {
    if (lane == 0) {
      int issued = 0;
      // Bulk L2 prefetch of a tile's z rows and x block (each one contiguous
      // range): the row warps then read them from L2 instead of DRAM, which
      // their few loads in flight could not keep busy.
      auto prefetch_tile = [&](int tile) {
        const int jb = tile % p.njb;
        const long long p0 = (long long)(tile / p.njb) * n + jb * 128;
        bulk_prefetch_l2(static_cast<const float*>(p.z) + p0 * 128,
                         (uint32_t)min(128, n - jb * 128) * 512u);
        const size_t xb = (size_t)128 * 128 * C::ESZ;
        bulk_prefetch_l2(static_cast<const uint8_t*>(p.x) + (size_t)tile * xb, (uint32_t)xb);
      };
      if (nmine > 0) prefetch_tile(blockIdx.x);
      for (int it = 0; it < nmine; ++it) {
        if (it + 1 < nmine) prefetch_tile(blockIdx.x + (it + 1) * gridDim.x);
        bool pushed = true;
        for (int q = 0; q < NLOADS; ++q) {
          const int nc = q / C::NKA, ka = q % C::NKA;
          if (!wring_push<kStrict>(ring, it * NLOADS + q, &w_hi, &w_lo, ka * C::KATOM, nc * 128,
                                   g)) {
            pushed = false;
            break;
          }
          ++issued;
        }
        if (!pushed) break;
      }
      if (g.aborted()) wring_drain(ring, issued, abort_flag);
    }
  } else {
    if (lane == 0) {
      const uint32_t idesc = kStrict ? idesc_tf32(128, 128) : idesc_bf16(128, 128);
      const uint32_t a_hi = smem_u32(A), a_lo = smem_u32(A + C::A_SPLIT_BYTES);
      bool ok = true;
      for (int it = 0; it < nmine && ok; ++it) {
        const int b = it & 1;
        // TMEM buffer b was read by the epilogue of tile it-2
        if (it >= 2 && !mbar_wait(&tfree[b], ((it - 2) >> 1) & 1, g, 8)) {
          ok = false;
          break;
        }
        for (int nc = 0; nc < 2 && ok; ++nc) {
          if (!mbar_wait(a_full, nc, g, 4)) {
            ok = false;
            break;
          }
          tc_fence_after();
          for (int ka = 0; ka < C::NKA; ++ka) {
            const int q = it * NLOADS + nc * C::NKA + ka;
            const uint32_t w = wring_wait(ring, q, g);
            if (!w) {
              ok = false;
              break;
            }
            mma_k_atom<kStrict>(tmem + b * 256 + nc * 128, a_hi + ka * C::ATOM_BYTES,
                                a_lo + ka * C::ATOM_BYTES, w, w + C::ATOM_BYTES, idesc, ka == 0);
            wring_release(ring, q);
          }
          if (ok) umma_commit(gdone);
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
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ----------------------------------------------------------------------------
// weight packing: concatenate up to 4 [rows][128] FP32 matrices and split
// them into tf32 hi/lo (strict) or convert to BF16 (fast).
// ----------------------------------------------------------------------------
__global__ void pack_weights_kernel(PackSrc src, void* hi, void* lo, int strict) {
  const int total = src.count * src.rows_each * 128;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int mat = i / (src.rows_each * 128);
    const int off = i - mat * src.rows_each * 128;
    const float v = src.m[mat][off];
    if (strict) {
      float h, l;
      split_tf32(v, h, l);
      static_cast<float*>(hi)[i] = h;
      static_cast<float*>(lo)[i] = l;
    } else {
      static_cast<__nv_bfloat16*>(hi)[i] = __float2bfloat16_rn(v);
    }
  }
}

int pack_weights(const PackSrc& src, void* hi, void* lo, bool strict, cudaStream_t stream) {
  FPB_LAUNCH("pack_weights", stream,
             pack_weights_kernel<<<64, 256, 0, stream>>>(src, hi, lo, strict ? 1 : 0));
  return launch_status();
}

bool make_weight_maps(const void* hi, const void* lo, int rows, bool strict, CUtensorMap* mh,
                      CUtensorMap* ml) {
  const int esz = strict ? 4 : 2;
  const CUtensorMapDataType dt =
      strict ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t pitch = 128ull * esz;
  bool ok = make_map_3d(mh, hi, dt, 128, rows, 1, pitch, pitch * rows, 128 / esz, 128, 1);
  if (strict)
    ok = ok && make_map_3d(ml, lo, dt, 128, rows, 1, pitch, pitch * rows, 128 / esz, 128, 1);
  else
    *ml = *mh;
  return ok;
}

// workspace plan (shared by the size query and the call)
// ----------------------------------------------------------------------------
// phases (shared by the fused single-GPU call and the row-sharded calls)
// ----------------------------------------------------------------------------
int trimul_proj_run(const float* z_loc, const float* mask, int yrows, int ycols, int zcols,
                    int r0, bool transposed, const float* ln_w, const float* ln_b,
                    const float* w_a_p, const float* w_a_g, const float* w_b_p,
                    const float* w_b_g, float eps, void* a_hi, void* a_lo, void* b_hi,
                    void* b_lo, int ld, int plane_rows, bool strict, void* wp_hi, void* wp_lo,
                    int* status, cudaStream_t stream, int owners = 0, int rank = 0,
                    void* const* a_owner = nullptr, void* const* b_owner = nullptr) {
  int st = pack_weights(PackSrc{{w_a_p, w_a_g, w_b_p, w_b_g}, 4, 128}, wp_hi, wp_lo, strict,
                        stream);
  if (st) return st;
  CUtensorMap mph, mpl;
  if (!make_weight_maps(wp_hi, wp_lo, 512, strict, &mph, &mpl)) return kErrArg;
  // raw z rows of a tile (strict): [128 rows][32 channels] boxes, rows past
  // ycols zero-filled; transposed: tile rows are rows of z at column r
  CUtensorMap zm{};
  if (strict) {
    const uint64_t rowb = 128ull * 4, pitch = (uint64_t)zcols * rowb;
    const bool zok =
        transposed
            ? make_map_3d(&zm, z_loc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 128, yrows, ycols, rowb,
                          pitch, 32, 1, 128)
            : make_map_3d(&zm, z_loc, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 128, ycols, yrows, rowb,
                          pitch, 32, 128, 1);
    if (!zok) return kErrArg;
  }
  const size_t cs = (size_t)plane_rows * ld;
  // strict with no a_lo / b_lo: a / b written unsplit into the hi planes
  const int a_plain = (strict && a_lo == nullptr) ? 1 : 0;
  const int b_plain = (strict && b_lo == nullptr) ? 1 : 0;
  const int tiles = yrows * ((ycols + 127) / 128);
  TriMulProjArgs pa{z_loc, mask, yrows, ycols, zcols, r0,   eps,    ln_w,  ln_b,   a_hi,
                    a_lo,  b_hi, b_lo,  ld,    cs,    status, b_plain, tiles, a_plain};
  pa.owners = owners;
  pa.gch = owners ? 128 / owners : 0;
  pa.rank = rank;
  for (int d = 0; d < owners; ++d) {
    pa.a_out[d] = a_owner[d];
    pa.b_out[d] = b_owner[d];
  }
  const unsigned grid = (unsigned)(tiles < sm_count() ? tiles : sm_count());
  const int smem = strict ? proj_smem_bytes<true>() : proj_smem_bytes<false>();
  auto k = strict ? (transposed ? trimul_proj_kernel<true, true> : trimul_proj_kernel<true, false>)
                  : (transposed ? trimul_proj_kernel<false, true>
                                : trimul_proj_kernel<false, false>);
  if (int smem_st = set_max_smem(k, smem)) return smem_st;
  FPB_LAUNCH("trimul_proj", stream,
             k<<<grid, 320, smem, stream>>>(mph, mpl, zm, pa));
  return launch_status();
}

int trimul_finish_run(float* z_loc, int n, int rows, const void* x_blocked, const float* ln_in_w,
                      const float* ln_in_b, const float* w_g, const float* ln_out_w,
                      const float* ln_out_b, const float* w_z, float eps, bool add, bool strict,
                      void* wo_hi, void* wo_lo, int* status, cudaStream_t stream) {
  int st = pack_weights(PackSrc{{w_g, w_z, nullptr, nullptr}, 2, 128}, wo_hi, wo_lo, strict,
                        stream);
  if (st) return st;
  CUtensorMap moh, mol;
  if (!make_weight_maps(wo_hi, wo_lo, 256, strict, &moh, &mol)) return kErrArg;
  const int njb = (n + 127) / 128;
  const int out_tiles = rows * njb;
  TriMulOutArgs oa{z_loc, n, eps, eps, ln_in_w, ln_in_b, ln_out_w, ln_out_b, x_blocked, njb,
                   add ? 1 : 0, status, out_tiles};
  const int smem = strict ? out_smem_bytes<true>() : out_smem_bytes<false>();
  auto k = strict ? trimul_out_kernel<true> : trimul_out_kernel<false>;
  if (int smem_st = set_max_smem(k, smem)) return smem_st;
  const unsigned grid = (unsigned)min(out_tiles, sm_count());
  FPB_LAUNCH("trimul_out", stream, k<<<grid, 192, smem, stream>>>(moh, mol, oa));
  return launch_status();
}

int trimul_contract_run(const void* a_hi, const void* a_lo, int m, int a_plane_rows,
                        const void* b_hi, const void* b_lo, int nn, int b_chunk_rows,
                        int b_chunks, size_t b_chunk_stride, int k, int ld, void* x_blocked,
                        bool strict, int* status, cudaStream_t stream, int channels = 128,
                        void* const* x_owner = nullptr, int owners = 0, int owner_rows = 0,
                        int ch_off = 0) {
  ContractOperands op{a_hi, a_lo, b_hi, b_lo, ld, (size_t)a_plane_rows * ld,
                      (size_t)b_chunk_rows * ld,
                      m, nn, k, b_chunk_rows, b_chunks, b_chunk_stride, channels, strict};
  ContractArgs ca{};
  ca.out = x_blocked;
  ca.out_bf16 = strict ? 0 : 1;
  ca.status = status;
  ca.blocked = 1;
  ca.njb = (nn + 127) / 128;
  ca.bchannels = channels;
  ca.owners = owners;
  ca.owner_rows = owner_rows;
  ca.ch_off = ch_off;
  for (int d = 0; d < owners; ++d) ca.outs[d] = x_owner[d];
  return launch_contract(op, ca, stream);
}

template <class Alloc>
struct TriMulPlan {
  void *wp_hi = nullptr, *wp_lo = nullptr, *wo_hi = nullptr, *wo_lo = nullptr;
  void *a_hi = nullptr, *a_lo = nullptr, *b_hi = nullptr, *b_lo = nullptr, *x = nullptr;
  int ld = 0, njb = 0;
  size_t cs = 0;
  void plan(Alloc& al, int n, bool strict) {
    auto takef = [&](size_t c) -> void* { return al.template take<float>(c); };
    auto takeh = [&](size_t c) -> void* { return al.template take<__nv_bfloat16>(c); };
    auto take = [&](size_t c) -> void* { return strict ? takef(c) : takeh(c); };
    wp_hi = take(512 * 128);
    if (strict) wp_lo = take(512 * 128);
    wo_hi = take(256 * 128);
    if (strict) wo_lo = take(256 * 128);
    ld = padded_ld(n, strict ? 4 : 2);
    cs = (size_t)n * ld;
    a_hi = take(128 * cs);
    b_hi = take(128 * cs);
    if (strict) {
      a_lo = take(128 * cs);
      b_lo = take(128 * cs);
    }
    njb = (n + 127) / 128;
    x = take((size_t)n * njb * 128 * 128);  // blocked [n][njb][128 c][128 j]
  }
};

// packed weights of one phase call (projection: 512 rows; finish: 256 rows)
template <class Alloc>
void plan_weights(Alloc& al, bool strict, int rows, void** hi, void** lo) {
  auto take = [&](size_t c) -> void* {
    return strict ? (void*)al.template take<float>(c) : (void*)al.template take<__nv_bfloat16>(c);
  };
  *hi = take((size_t)rows * 128);
  *lo = strict ? take((size_t)rows * 128) : nullptr;
}

}  // namespace fpb

using namespace fpb;

extern "C" size_t fpb_trimul_workspace_size(int n, int c_z, int precision) {
  if (n <= 0 || c_z != 128 || (precision != 0 && precision != 1)) return 0;
  WsCounter cnt;
  TriMulPlan<WsCounter> pl;
  pl.plan(cnt, n, precision == 0);
  return cnt.used;
}

extern "C" int fpb_trimul(float* z, const float* mask, int n, int c_z, const float* ln_in_w,
                          const float* ln_in_b, const float* w_a_p, const float* w_a_g,
                          const float* w_b_p, const float* w_b_g, const float* w_g,
                          const float* ln_out_w, const float* ln_out_b, const float* w_z,
                          float eps, int outgoing, int add, int precision, void* workspace,
                          size_t workspace_bytes, cudaStream_t stream) {
  if (!z || !ln_in_w || !ln_in_b || !w_a_p || !w_a_g || !w_b_p || !w_b_g || !w_g || !ln_out_w ||
      !ln_out_b || !w_z || !workspace)
    return kErrArg;
  if (c_z != 128 || n <= 0) return kErrShape;
  if (precision != 0 && precision != 1) return kErrArg;
  if (!aligned16(z) || !aligned16(workspace) || !aligned16(ln_in_w) || !aligned16(ln_in_b))
    return kErrAlign;
  if (workspace_bytes < fpb_trimul_workspace_size(n, c_z, precision)) return kErrWorkspace;
  const bool strict = precision == 0;
  WsCursor cur(workspace, workspace_bytes);
  TriMulPlan<WsCursor> pl;
  pl.plan(cur, n, strict);
  if (!cur.ok) return kErrWorkspace;
  int* status = static_cast<int*>(workspace);
  if (reset_status(workspace, stream)) return kErrCuda;
  int st = trimul_proj_run(z, mask, n, n, n, 0, !outgoing, ln_in_w, ln_in_b, w_a_p, w_a_g, w_b_p,
                           w_b_g, eps, pl.a_hi, pl.a_lo, pl.b_hi, pl.b_lo, pl.ld, n, strict,
                           pl.wp_hi, pl.wp_lo, status, stream);
  if (st) return st;
  st = trimul_contract_run(pl.a_hi, pl.a_lo, n, n, pl.b_hi, pl.b_lo, n, n, 1, 0, n, pl.ld, pl.x,
                           strict, status, stream);
  if (st) return st;
  return trimul_finish_run(z, n, n, pl.x, ln_in_w, ln_in_b, w_g, ln_out_w, ln_out_b, w_z, eps,
                           add != 0, strict, pl.wo_hi, pl.wo_lo, status, stream);
}

// ---------------------------------------------------------------- row-sharded phases
extern "C" size_t fpb_trimul_shard_workspace_size(int precision) {
  if (precision != 0 && precision != 1) return 0;
  WsCounter cnt;
  void *h, *l;
  plan_weights(cnt, precision == 0, 512, &h, &l);
  return cnt.used;
}

extern "C" size_t fpb_trimul_plane_ld(int cols, int precision) {
  return (size_t)padded_ld(cols, precision == 0 ? 4 : 2);
}

extern "C" int fpb_trimul_shard_proj(const float* z_loc, const float* mask, int n, int rows,
                                     int r0, int transposed, const float* ln_in_w,
                                     const float* ln_in_b, const float* w_a_p, const float* w_a_g,
                                     const float* w_b_p, const float* w_b_g, float eps, void* a_hi,
                                     void* a_lo, void* b_hi, void* b_lo, int ld, int plane_rows,
                                     int precision, void* workspace, size_t workspace_bytes,
                                     cudaStream_t stream) {
  if (!z_loc || !a_hi || !b_hi || !workspace || !ln_in_w || !ln_in_b || !w_a_p || !w_a_g ||
      !w_b_p || !w_b_g)
    return kErrArg;
  if (precision != 0 && precision != 1) return kErrArg;
  const bool strict = precision == 0;
  // strict: a_lo / b_lo null writes a / b unsplit (FP32) into the hi planes
  if (n <= 0 || rows <= 0 || r0 < 0 || r0 + rows > n) return kErrShape;
  const int yrows = transposed ? n : rows;
  const int ycols = transposed ? rows : n;
  if (plane_rows < yrows) return kErrShape;
  if (ld < ycols || ld % (strict ? 32 : 64)) return kErrAlign;
  if (!aligned16(z_loc) || !aligned16(workspace) || !aligned16(ln_in_w) || !aligned16(ln_in_b))
    return kErrAlign;
  if (workspace_bytes < fpb_trimul_shard_workspace_size(precision)) return kErrWorkspace;
  WsCursor cur(workspace, workspace_bytes);
  void *wh, *wl;
  plan_weights(cur, strict, 512, &wh, &wl);
  if (reset_status(workspace, stream)) return kErrCuda;
  // outgoing: y = z_loc (rows x n); incoming: y = z_loc^T (n x rows)
  return trimul_proj_run(z_loc, mask, yrows, ycols, n, r0, transposed != 0, ln_in_w, ln_in_b,
                         w_a_p, w_a_g, w_b_p, w_b_g, eps, a_hi, a_lo, b_hi, b_lo, ld, plane_rows,
                         strict, wh, wl, static_cast<int*>(workspace), stream);
}

extern "C" int fpb_trimul_shard_proj_scatter(
    const float* z_loc, const float* mask, int n, int rows, int r0, int transposed,
    const float* ln_in_w, const float* ln_in_b, const float* w_a_p, const float* w_a_g,
    const float* w_b_p, const float* w_b_g, float eps, void* const* a_owner,
    void* const* b_owner, int owners, int rank, int ld, int plane_rows, int precision,
    void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!z_loc || !a_owner || !b_owner || !workspace || !ln_in_w || !ln_in_b || !w_a_p ||
      !w_a_g || !w_b_p || !w_b_g)
    return kErrArg;
  if (precision != 0 && precision != 1) return kErrArg;
  const bool strict = precision == 0;
  if (owners <= 0 || owners > 16 || 128 % owners || rank < 0 || rank >= owners) return kErrShape;
  for (int d = 0; d < owners; ++d)
    if (!a_owner[d] || !b_owner[d] || !aligned16(a_owner[d]) || !aligned16(b_owner[d]))
      return kErrArg;
  if (n <= 0 || rows <= 0 || r0 < 0 || r0 + rows > n) return kErrShape;
  const int yrows = transposed ? n : rows;
  const int ycols = transposed ? rows : n;
  if (plane_rows < yrows) return kErrShape;
  if (ld < ycols || ld % (strict ? 32 : 64)) return kErrAlign;
  if (!aligned16(z_loc) || !aligned16(workspace) || !aligned16(ln_in_w) || !aligned16(ln_in_b))
    return kErrAlign;
  if (workspace_bytes < fpb_trimul_shard_workspace_size(precision)) return kErrWorkspace;
  WsCursor cur(workspace, workspace_bytes);
  void *wh, *wl;
  plan_weights(cur, strict, 512, &wh, &wl);
  if (reset_status(workspace, stream)) return kErrCuda;
  // a / b unsplit (the receivers split their operand while gathering it)
  return trimul_proj_run(z_loc, mask, yrows, ycols, n, r0, transposed != 0, ln_in_w, ln_in_b,
                         w_a_p, w_a_g, w_b_p, w_b_g, eps, a_owner[rank], nullptr, b_owner[rank],
                         nullptr, ld, plane_rows, strict, wh, wl, static_cast<int*>(workspace),
                         stream, owners, rank, a_owner, b_owner);
}

extern "C" int fpb_trimul_group_contract(const void* a_hi, const void* a_lo, int m,
                                         int a_plane_rows, const void* b_hi, const void* b_lo,
                                         int nn, int b_chunk_rows, int b_chunks,
                                         size_t b_chunk_stride, int k, int ld, int channels,
                                         void* x_blocked, int precision, void* workspace,
                                         size_t workspace_bytes, cudaStream_t stream) {
  if (!a_hi || !b_hi || !x_blocked || !workspace) return kErrArg;
  if (precision != 0 && precision != 1) return kErrArg;
  const bool strict = precision == 0;
  if (strict && (!a_lo || !b_lo)) return kErrArg;
  if (m <= 0 || nn <= 0 || k <= 0 || b_chunk_rows <= 0 || b_chunks <= 0 || a_plane_rows < m ||
      (long long)b_chunk_rows * b_chunks < nn || channels <= 0 || channels > 128)
    return kErrShape;
  if (workspace_bytes < kWsHeader || !aligned16(workspace)) return kErrWorkspace;
  if (reset_status(workspace, stream)) return kErrCuda;
  return trimul_contract_run(a_hi, a_lo, m, a_plane_rows, b_hi, b_lo, nn, b_chunk_rows, b_chunks,
                             b_chunk_stride, k, ld, x_blocked, strict,
                             static_cast<int*>(workspace), stream, channels);
}

extern "C" int fpb_trimul_group_contract_scatter(
    const void* a_hi, const void* a_lo, int m, int a_plane_rows, const void* b_hi,
    const void* b_lo, int nn, int b_chunk_rows, int b_chunks, size_t b_chunk_stride, int k, int ld,
    int channels, void* const* x_owner, int owners, int owner_rows, int ch_off, int precision,
    void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!a_hi || !b_hi || !x_owner || !workspace) return kErrArg;
  if (precision != 0 && precision != 1) return kErrArg;
  const bool strict = precision == 0;
  if (strict && (!a_lo || !b_lo)) return kErrArg;
  if (m <= 0 || nn <= 0 || k <= 0 || b_chunk_rows <= 0 || b_chunks <= 0 || a_plane_rows < m ||
      (long long)b_chunk_rows * b_chunks < nn || channels <= 0 || channels > 128)
    return kErrShape;
  if (owners <= 0 || owners > 16 || owner_rows <= 0 || (long long)owners * owner_rows < m ||
      ch_off < 0 || ch_off + channels > 128)
    return kErrShape;
  for (int d = 0; d < owners; ++d)
    if ((long long)d * owner_rows < m && (!x_owner[d] || !aligned16(x_owner[d]))) return kErrArg;
  if (workspace_bytes < kWsHeader || !aligned16(workspace)) return kErrWorkspace;
  if (reset_status(workspace, stream)) return kErrCuda;
  return trimul_contract_run(a_hi, a_lo, m, a_plane_rows, b_hi, b_lo, nn, b_chunk_rows, b_chunks,
                             b_chunk_stride, k, ld, x_owner[0], strict,
                             static_cast<int*>(workspace), stream, channels, x_owner, owners,
                             owner_rows, ch_off);
}

extern "C" int fpb_trimul_shard_contract(const void* a_hi, const void* a_lo, int m,
                                         int a_plane_rows, const void* b_hi, const void* b_lo,
                                         int nn, int b_chunk_rows, int b_chunks,
                                         size_t b_chunk_stride, int k, int ld, void* x_blocked,
                                         int precision, void* workspace, size_t workspace_bytes,
                                         cudaStream_t stream) {
  return fpb_trimul_group_contract(a_hi, a_lo, m, a_plane_rows, b_hi, b_lo, nn, b_chunk_rows,
                                   b_chunks, b_chunk_stride, k, ld, 128, x_blocked, precision,
                                   workspace, workspace_bytes, stream);
}

extern "C" int fpb_trimul_shard_finish(float* z_loc, int n, int rows, const void* x_blocked,
                                       const float* ln_in_w, const float* ln_in_b,
                                       const float* w_g, const float* ln_out_w,
                                       const float* ln_out_b, const float* w_z, float eps, int add,
                                       int precision, void* workspace, size_t workspace_bytes,
                                       cudaStream_t stream) {
  if (!z_loc || !x_blocked || !workspace || !ln_in_w || !ln_in_b || !w_g || !ln_out_w ||
      !ln_out_b || !w_z)
    return kErrArg;
  if (precision != 0 && precision != 1) return kErrArg;
  if (n <= 0 || rows <= 0) return kErrShape;
  if (!aligned16(z_loc) || !aligned16(workspace) || !aligned16(ln_in_w) || !aligned16(ln_in_b))
    return kErrAlign;
  const bool strict = precision == 0;
  if (workspace_bytes < fpb_trimul_shard_workspace_size(precision)) return kErrWorkspace;
  WsCursor cur(workspace, workspace_bytes);
  void *wh, *wl;
  plan_weights(cur, strict, 256, &wh, &wl);
  if (reset_status(workspace, stream)) return kErrCuda;
  return trimul_finish_run(z_loc, n, rows, x_blocked, ln_in_w, ln_in_b, w_g, ln_out_w, ln_out_b,
                           w_z, eps, add != 0, strict, wh, wl, static_cast<int*>(workspace),
                           stream);
}

// Exact tf32 split of FP32 values: hi = x with the low 13 mantissa bits
// cleared, lo = x - hi. hi may alias src (in-place split).
namespace fpb {
__global__ void split_tf32_kernel(const float* src, float* hi, float* lo, size_t count) {
  const size_t n4 = count / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
       i += (size_t)gridDim.x * blockDim.x) {
    const float4 x = reinterpret_cast<const float4*>(src)[i];
    float4 h, l;
    split_tf32(x.x, h.x, l.x);
    split_tf32(x.y, h.y, l.y);
    split_tf32(x.z, h.z, l.z);
    split_tf32(x.w, h.w, l.w);
    reinterpret_cast<float4*>(hi)[i] = h;
    reinterpret_cast<float4*>(lo)[i] = l;
  }
  for (size_t i = n4 * 4 + blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count;
       i += (size_t)gridDim.x * blockDim.x) {
    float h, l;
    split_tf32(src[i], h, l);
    hi[i] = h;
    lo[i] = l;
  }
}
}  // namespace fpb

extern "C" int fpb_split_tf32(const float* src, void* hi, void* lo, size_t count,
                              cudaStream_t stream) {
  if (!src || !hi || !lo) return kErrArg;
  if (!aligned16(src) || !aligned16(hi) || !aligned16(lo)) return kErrAlign;
  if (count == 0) return kOk;
  const unsigned blocks = (unsigned)min((size_t)sm_count() * 8, (count / 4 + 255) / 256 + 1);
  FPB_LAUNCH("split_tf32", stream,
             split_tf32_kernel<<<blocks, 256, 0, stream>>>(src, static_cast<float*>(hi),
                                                           static_cast<float*>(lo), count));
  return launch_status();
}

// ----------------------------------------------------------------------------
// channel-group gather of the received TriMul planes (channel-sharded
// exchange): src [W][G][R][src_ld] -> the contraction operand, split into
// hi/lo (strict) or copied (fast) in the same pass.
//   rows mode: dst[c][r * R + i][k]       = src[r][c][i][k], k < seg
//   cols mode: dst[c][i][r * seg + k]     = src[r][c][i][k], k < seg
// One work unit = 4 consecutive k of one (r, c, i) segment.
// ----------------------------------------------------------------------------
namespace fpb {
template <bool kStrict>
__global__ void group_gather_kernel(const void* __restrict__ src, int W, int G, int R,
                                    int src_ld, int seg, int cols_mode, void* __restrict__ hi,
                                    void* __restrict__ lo, int dst_ld) {
  const int s4 = seg / 4;
  const size_t units = (size_t)W * G * R * s4;
  for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < units;
       u += (size_t)gridDim.x * blockDim.x) {
    const int k = (int)(u % s4) * 4;
    size_t rest = u / s4;
    const int i = (int)(rest % R);
    rest /= R;
    const int c = (int)(rest % G);
    const int r = (int)(rest / G);
    const size_t so = (((size_t)r * G + c) * R + i) * src_ld + k;
    const size_t dof = cols_mode ? ((size_t)c * R + i) * dst_ld + (size_t)r * seg + k
                                 : ((size_t)c * W * R + (size_t)r * R + i) * dst_ld + k;
    if constexpr (kStrict) {
      const float4 x = *reinterpret_cast<const float4*>(static_cast<const float*>(src) + so);
      float4 h, l;
      split_tf32(x.x, h.x, l.x);
      split_tf32(x.y, h.y, l.y);
      split_tf32(x.z, h.z, l.z);
      split_tf32(x.w, h.w, l.w);
      *reinterpret_cast<float4*>(static_cast<float*>(hi) + dof) = h;
      *reinterpret_cast<float4*>(static_cast<float*>(lo) + dof) = l;
    } else {
      *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(hi) + dof) =
          *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(src) + so);
    }
  }
}
}  // namespace fpb

extern "C" int fpb_trimul_group_gather(const void* src, int world, int channels, int rows,
                                       int src_ld, int seg, int cols_mode, void* dst_hi,
                                       void* dst_lo, int dst_ld, int precision,
                                       cudaStream_t stream) {
  if (!src || !dst_hi) return kErrArg;
  if (precision != 0 && precision != 1) return kErrArg;
  const bool strict = precision == 0;
  if (strict && !dst_lo) return kErrArg;
  if (world <= 0 || channels <= 0 || rows <= 0 || seg <= 0 || seg > src_ld) return kErrShape;
  if (cols_mode ? dst_ld < (long long)world * seg : dst_ld < seg) return kErrShape;
  if (seg % 4 || src_ld % 4 || dst_ld % 4) return kErrAlign;
  if (!aligned16(src) || !aligned16(dst_hi) || (strict && !aligned16(dst_lo))) return kErrAlign;
  const size_t units = (size_t)world * channels * rows * (seg / 4);
  const unsigned blocks = (unsigned)min((size_t)sm_count() * 8, (units + 255) / 256);
  if (strict)
    FPB_LAUNCH("group_gather", stream,
               (group_gather_kernel<true><<<blocks, 256, 0, stream>>>(
                   src, world, channels, rows, src_ld, seg, cols_mode, dst_hi, dst_lo, dst_ld)));
  else
    FPB_LAUNCH("group_gather", stream,
               (group_gather_kernel<false><<<blocks, 256, 0, stream>>>(
                   src, world, channels, rows, src_ld, seg, cols_mode, dst_hi, nullptr, dst_ld)));
  return launch_status();
}
