// Pair transition (SwiGLU, 4x expansion), fused on sm_100a.
//
// Reference: Protenix Transition as dispatched by
// python/fireprot/backends/amd/recycle.py:203-227,360 (projection kernel
// kernels/amd/fireprot_amd_ops.cu:1106-1183):
//   x = LN(z); h = silu(x Wa^T) * (x Wb^T)   (Wa, Wb [512,128])
//   z <- z + h Wout^T                        (Wout [128,512])
//
// One kernel per 128-row tile. The hidden dimension is processed in chunks of
// HC = one 128-byte K atom (32 fp32 / 64 bf16): GEMM 1 computes [a_c | b_c]
// (N = 2*HC) into a double-buffered TMEM region, the row threads form
// h_c = silu(a_c) * b_c and write it to shared memory as the A operand of
// GEMM 2, which accumulates h_c Wout[:, c]^T into a 128-column TMEM
// accumulator. The 4x-wide intermediate never reaches HBM.
#include "../../include/fireprot_b200.h"
#include "kernels.h"
#include "rowgemm.cuh"

namespace fpb {

template <bool kStrict>
struct TransCfg {
  using R = RowCfg<kStrict>;
  // hidden chunk: 64 columns in both modes (two fp32 K atoms / one bf16 atom).
  // Each chunk pays a fixed latency chain (GEMM-1 commit, TMEM read, SwiGLU,
  // shared-memory store, barrier round trips), so fewer, wider chunks keep
  // the tensor pipe busier; GEMM 1 is then N = 128 (cheaper per column than
  // N = 64 in the TS form).
  static constexpr int NHA = kStrict ? 2 : 1;  // K atoms of GEMM 2 per chunk
  static constexpr int HC = NHA * R::KATOM;    // 64
  static constexpr int NCH = 512 / HC;         // 8 chunks
  static constexpr int G1N = 2 * HC;           // GEMM 1 width (a_c | b_c) = 128
  static constexpr int G1_STAGE = G1N * 128 * R::NSPLIT;   // bytes of one GEMM-1 W stage
  static constexpr int G2_STAGE = 128 * 128 * R::NSPLIT;   // bytes of one GEMM-2 W stage (one atom)
  static constexpr int STAGE = G1_STAGE > G2_STAGE ? G1_STAGE : G2_STAGE;
  static constexpr int STAGES = 5;
  static constexpr int H_ATOM = R::NSPLIT * R::ATOM_BYTES;  // one K atom of H (hi | lo)
  static constexpr int H_BYTES = NHA * H_ATOM;              // one chunk of H
  // strict: the 512 TMEM columns and 227 KB of shared memory hold one GEMM-1
  // buffer and one H tile; fast: two of each
  static constexpr int G1_BUFS = kStrict ? 1 : 2;
  static constexpr int H_BUFS = kStrict ? 1 : 2;
  // TMEM: A = LN(z) (tf32 hi | lo: 256 columns; bf16 pairs: 64), the GEMM-1
  // buffer(s), the GEMM-2 accumulator (128)
  static constexpr uint32_t kA_LO = 128;
  static constexpr uint32_t kG1 = kStrict ? 256 : 64;
  static constexpr uint32_t kAcc = kG1 + G1_BUFS * G1N;
  static constexpr int TMEM_COLS = 512;
  static_assert(kAcc + 128 <= TMEM_COLS, "TMEM budget");
  static constexpr int SMEM =
      tmem_safe_smem(H_BUFS * H_BYTES + STAGES * STAGE + 1024 + 256 + 1024, TMEM_COLS);
};

struct TransArgs {
  float* z;
  float* delta;  // when non-null: write the update here and leave z unchanged
  int n_rows;
  float eps;
  const float* ln_w;
  const float* ln_b;
  int* status;
};

// One CTA per 128-row tile. The LayerNorm'd tile lives in TMEM (thread t =
// row t normalises its own row and stores it as the A operand of GEMM 1), so
// shared memory holds only the SwiGLU tile(s) H and a 5-stage weight ring:
//   GEMM 1 (chunk c): [a_c | b_c] = A [Wa_c; Wb_c]^T     (A from TMEM)
//   row threads:      H = silu(a_c) * b_c -> shared memory (A operand)
//   GEMM 2:           acc += H Wout_c^T
// The MMA warp issues GEMM 1(c+1) once the row threads have read GEMM 1(c)
// out of TMEM, and GEMM 2(c) once H(c) is written, so the tensor pipe runs
// GEMM 1(c+1), GEMM 2(c), GEMM 1(c+2), ... while the row threads work on
// chunk c+1. Fast mode double-buffers GEMM 1 and H as well.
template <bool kStrict>
__global__ void __launch_bounds__(192, 1)
    transition_kernel(const __grid_constant__ CUtensorMap w1_hi,
                      const __grid_constant__ CUtensorMap w1_lo,
                      const __grid_constant__ CUtensorMap w2_hi,
                      const __grid_constant__ CUtensorMap w2_lo, TransArgs p) {
  using R = RowCfg<kStrict>;
  using C = TransCfg<kStrict>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* H = smem;                 // [H_BUFS][H_BYTES]
  uint8_t* W = H + C::H_BUFS * C::H_BYTES;
  float* lnp = reinterpret_cast<float*>(W + C::STAGES * C::STAGE);  // [2][128]
  uint64_t* bars = reinterpret_cast<uint64_t*>(lnp + 256);
  uint64_t* wfull = bars;
  uint64_t* wempty = wfull + C::STAGES;
  uint64_t* a_full = wempty + C::STAGES;
  uint64_t* g1_full = a_full + 1;   // [2]
  uint64_t* g1_free = g1_full + 2;  // [2]
  uint64_t* h_full = g1_free + 2;  // [2]
  uint64_t* h_free = h_full + 2;   // [2]
  uint64_t* done = h_free + 2;
  uint64_t* drain = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long rows = p.n_rows;
  const int ntiles = (int)((rows + 127) / 128);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], 1);
    }
    mbar_init(a_full, 128);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&g1_full[b], 1);
      mbar_init(&g1_free[b], 128);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&h_full[b], 128);
      mbar_init(&h_free[b], 1);
    }
    mbar_init(done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < 128) {
    lnp[threadIdx.x] = p.ln_w[threadIdx.x];
    lnp[128 + threadIdx.x] = p.ln_b[threadIdx.x];
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

  // Weight-load sequence shared by the TMA and MMA threads:
  // G1(0), then for c = 0..NCH-1: [G1(c+1)], G2(c). G1 chunk = R::NKA loads.
  if (warp < 4) {
    const int t = warp * 32 + lane;
    const uint32_t lrow = tmem + ((uint32_t)(warp * 32) << 16);  // this thread's TMEM lane
    // residual epilogue of a finished tile (thread t owns its row pr)
    auto epilogue = [&](long long pr, int it_done) -> bool {
      if (!mbar_wait(done, it_done & 1, g, 3)) return false;
      tc_fence_after();
      const long long rsafe = pr < rows ? pr : 0;
      float4* zrow = reinterpret_cast<float4*>(p.z) + rsafe * 32;
      float4* drow = p.delta ? reinterpret_cast<float4*>(p.delta) + rsafe * 32 : zrow;
      const bool residual = p.delta == nullptr;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        float4 zc[8];
#pragma unroll
        for (int v4 = 0; v4 < 8; ++v4)
          zc[v4] = (residual && pr < rows) ? zrow[cc * 8 + v4] : make_float4(0.f, 0.f, 0.f, 0.f);
        float yv[32];
        tmem_row32(tmem + C::kAcc, warp, cc * 32, yv);
        if (pr < rows) {
#pragma unroll
          for (int v4 = 0; v4 < 8; ++v4) {
            float4 o = zc[v4];
            o.x += yv[4 * v4];
            o.y += yv[4 * v4 + 1];
            o.z += yv[4 * v4 + 2];
            o.w += yv[4 * v4 + 3];
            drow[cc * 8 + v4] = o;
          }
        }
      }
      tc_fence_before();  // acc read before the next tile's GEMM 2 writes it
      return true;
    };
    bool ok = true;
    int it = 0;
    long long pprev = 0;
    // persistent: tiles blockIdx.x, + gridDim.x, ... Per tile: LayerNorm into
    // A (free once GEMM 1 of the previous tile's last chunk has retired, which
    // this thread has waited for), the previous tile's epilogue (while GEMM 1
    // of this tile runs), then the SwiGLU chunks
#pragma unroll 1
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
    const long long pr = (long long)tile * 128 + t;
    {
      // ---- A = LN(z row t) into TMEM: one row per thread, all loads first
      float x[128];
      const float4* zr = reinterpret_cast<const float4*>(p.z) + (pr < rows ? pr : 0) * 32;
#pragma unroll
      for (int v4 = 0; v4 < 32; ++v4) {
        const float4 v = pr < rows ? __ldg(zr + v4) : make_float4(0.f, 0.f, 0.f, 0.f);
        x[4 * v4] = v.x;
        x[4 * v4 + 1] = v.y;
        x[4 * v4 + 2] = v.z;
        x[4 * v4 + 3] = v.w;
      }
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 128; ++c) s4[c & 3] += x[c];
      const float mean = ((s4[0] + s4[1]) + (s4[2] + s4[3])) * (1.0f / 128.0f);
      float q4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        const float d = x[c] - mean;
        q4[c & 3] += d * d;
      }
      const float rs =
          rsqrtf(((q4[0] + q4[1]) + (q4[2] + q4[3])) * (1.0f / 128.0f) + p.eps);
#pragma unroll
      for (int c = 0; c < 128; ++c) x[c] = (x[c] - mean) * rs * lnp[c] + lnp[128 + c];
      if constexpr (kStrict) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t hv[32], lv[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            float h, l;
            split_tf32(x[q * 32 + e], h, l);
            hv[e] = __float_as_uint(h);
            lv[e] = __float_as_uint(l);
          }
          tmem_st32(lrow + q * 32, hv);
          tmem_st32(lrow + C::kA_LO + q * 32, lv);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t pk[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(x[q * 64 + 2 * e], x[q * 64 + 2 * e + 1]);
            pk[e] = *reinterpret_cast<uint32_t*>(&b2);
          }
          tmem_st32(lrow + q * 32, pk);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(a_full);
    }
    if (it > 0 && !epilogue(pprev, it - 1)) {
      ok = false;
      break;
    }
#pragma unroll 1
    for (int c = 0; c < C::NCH && ok; ++c) {
      const int cg = it * C::NCH + c;  // chunk index over this CTA's tiles
      const int b = cg % C::G1_BUFS;
      if (!mbar_wait(&g1_full[b], (cg / C::G1_BUFS) & 1, g, 31)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float hv[C::HC];
#pragma unroll
      for (int q = 0; q < C::HC / 32; ++q) {
        float av[32], bv[32];
        tmem_row32(tmem + C::kG1 + b * C::G1N, warp, q * 32, av);
        tmem_row32(tmem + C::kG1 + b * C::G1N, warp, C::HC + q * 32, bv);
#pragma unroll
        for (int e = 0; e < 32; ++e) hv[q * 32 + e] = av[e] * sigmoidf_(av[e]) * bv[e];
      }
      tc_fence_before();
      mbar_arrive(&g1_free[b]);
      // H buffer hb was read by GEMM 2 of chunk c - H_BUFS
      const int hb = cg % C::H_BUFS;
      if (cg >= C::H_BUFS &&
          !mbar_wait(&h_free[hb], ((cg - C::H_BUFS) / C::H_BUFS) & 1, g, 32)) {
        ok = false;
        break;
      }
      // H row t: HC elements over NHA K atoms
#pragma unroll
      for (int e = 0; e < C::HC; e += 4) {
        uint8_t* dst = H + hb * C::H_BYTES + (e / R::KATOM) * C::H_ATOM +
                       sw128_offset(t, (e % R::KATOM) * R::ESZ);
        if constexpr (kStrict) {
          float h0, l0, h1, l1, h2, l2, h3, l3;
          split_tf32(hv[e], h0, l0);
          split_tf32(hv[e + 1], h1, l1);
          split_tf32(hv[e + 2], h2, l2);
          split_tf32(hv[e + 3], h3, l3);
          *reinterpret_cast<float4*>(dst) = make_float4(h0, h1, h2, h3);
          *reinterpret_cast<float4*>(dst + R::ATOM_BYTES) = make_float4(l0, l1, l2, l3);
        } else {
          __nv_bfloat162 x0 = __floats2bfloat162_rn(hv[e], hv[e + 1]);
          __nv_bfloat162 x1 = __floats2bfloat162_rn(hv[e + 2], hv[e + 3]);
          uint2 w;
          w.x = *reinterpret_cast<uint32_t*>(&x0);
          w.y = *reinterpret_cast<uint32_t*>(&x1);
          *reinterpret_cast<uint2*>(dst) = w;
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&h_full[hb]);
    }
      pprev = pr;
    }  // tiles
    if (ok && it > 0) (void)epilogue(pprev, it - 1);
  } else if (warp == 4) {
    if (lane == 0) {
      int seq = 0;
      bool ok = true;
      auto push = [&](bool g2, int c, int atom) -> bool {
        const int s = seq % C::STAGES;
        const uint32_t ph = (seq / C::STAGES) & 1;
        if (seq >= C::STAGES && !mbar_wait(&wempty[s], ph ^ 1, g, 33)) return false;
        uint8_t* st = W + s * C::STAGE;
        if (g2) {
          const int k0 = c * C::HC + atom * R::KATOM;
          mbar_arrive_expect_tx(&wfull[s], C::G2_STAGE);
          tma_load_3d(st, &w2_hi, &wfull[s], k0, 0, 0);
          if constexpr (kStrict) tma_load_3d(st + R::ATOM_BYTES, &w2_lo, &wfull[s], k0, 0, 0);
        } else {
          mbar_arrive_expect_tx(&wfull[s], C::G1_STAGE);
          tma_load_3d(st, &w1_hi, &wfull[s], atom * R::KATOM, c * C::G1N, 0);
          if constexpr (kStrict)
            tma_load_3d(st + C::G1N * 128, &w1_lo, &wfull[s], atom * R::KATOM, c * C::G1N, 0);
        }
        ++seq;
        return true;
      };
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        for (int a = 0; a < R::NKA && ok; ++a) ok = push(false, 0, a);
        for (int c = 0; c < C::NCH && ok; ++c) {
          if (c + 1 < C::NCH)
            for (int a = 0; a < R::NKA && ok; ++a) ok = push(false, c + 1, a);
          for (int a = 0; a < C::NHA && ok; ++a) ok = push(true, c, a);
        }
      }
      if (g.aborted()) {
        for (int q = (seq > C::STAGES ? seq - C::STAGES : 0); q < seq; ++q)
          (void)mbar_wait(&wfull[q % C::STAGES], (q / C::STAGES) & 1, Guard{nullptr, abort_flag}, 0);
      }
    }
  } else {
    if (lane == 0) {
      const uint32_t id1 = kStrict ? idesc_tf32(128, C::G1N) : idesc_bf16(128, C::G1N);
      const uint32_t id2 = kStrict ? idesc_tf32(128, 128) : idesc_bf16(128, 128);
      const uint32_t h0 = smem_u32(H);
      int seq = 0;
      auto take = [&]() -> uint32_t {
        const int s = seq % C::STAGES;
        if (!mbar_wait(&wfull[s], (seq / C::STAGES) & 1, g, 34)) return 0;
        tc_fence_after();
        return smem_u32(W + s * C::STAGE);
      };
      auto release = [&]() {
        umma_commit(&wempty[seq % C::STAGES]);
        ++seq;
      };
      auto gemm1 = [&](int c) -> bool {
        const int b = c % C::G1_BUFS;
        if (c >= C::G1_BUFS &&
            !mbar_wait(&g1_free[b], ((c - C::G1_BUFS) / C::G1_BUFS) & 1, g, 35))
          return false;
        tc_fence_after();
        const uint32_t d = tmem + C::kG1 + b * C::G1N;
        for (int a = 0; a < R::NKA; ++a) {
          const uint32_t w = take();
          if (!w) return false;
          // A atom a from TMEM: 4 K steps of 8 tf32 / 16 bf16 (8 columns each)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint32_t acol = a * (R::KATOM * R::ESZ / 4) + kk * 8;
            const uint64_t dwh = umma_desc_sw128(w + kk * 32);
            const uint32_t acc = (a == 0 && kk == 0) ? 0u : 1u;
            if constexpr (kStrict) {
              const uint64_t dwl = umma_desc_sw128(w + C::G1N * 128 + kk * 32);
              umma_tf32_ts(d, tmem + acol, dwh, id1, acc);             // A_hi W_hi
              umma_tf32_ts(d, tmem + acol, dwl, id1, 1u);              // A_hi W_lo
              umma_tf32_ts(d, tmem + C::kA_LO + acol, dwh, id1, 1u);   // A_lo W_hi
            } else {
              umma_bf16_ts(d, tmem + acol, dwh, id1, acc);
            }
          }
          release();
        }
        umma_commit(&g1_full[b]);
        return true;
      };
      bool ok = true;
      int it = 0;
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++it) {
      const int cb = it * C::NCH;  // first chunk index of this tile
      ok = mbar_wait(a_full, it & 1, g, 36);
      if (ok) tc_fence_after();
      if (ok) ok = gemm1(cb);
      for (int c = 0; c < C::NCH && ok; ++c) {
        if (c + 1 < C::NCH && !(ok = gemm1(cb + c + 1))) break;
        const int hb = (cb + c) % C::H_BUFS;
        if (!mbar_wait(&h_full[hb], ((cb + c) / C::H_BUFS) & 1, g, 37)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int a = 0; a < C::NHA && ok; ++a) {
          const uint32_t w = take();
          if (!w) {
            ok = false;
            break;
          }
          const uint32_t h_hi = h0 + hb * C::H_BYTES + a * C::H_ATOM;
          mma_k_atom<kStrict>(tmem + C::kAcc, h_hi, h_hi + R::ATOM_BYTES, w, w + R::ATOM_BYTES,
                              id2, c == 0 && a == 0);
          release();
        }
        if (!ok) break;
        umma_commit(&h_free[hb]);
      }
      if (ok) umma_commit(done);
      }  // tiles
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
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Pack [Wa; Wb] chunk-interleaved: chunk c = rows Wa[c*HC..), Wb[c*HC..).
__global__ void pack_transition_w1(const float* __restrict__ wa, const float* __restrict__ wb,
                                   int hc, void* hi, void* lo, int strict) {
  const int total = 1024 * 128;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int row = i / 128, k = i % 128;
    const int c = row / (2 * hc), r = row % (2 * hc);
    const float v = r < hc ? wa[(c * hc + r) * 128 + k] : wb[(c * hc + r - hc) * 128 + k];
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

__global__ void pack_plain(const float* __restrict__ w, int count, void* hi, void* lo, int strict) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
    const float v = w[i];
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

template <class Alloc>
struct TransPlan {
  void *w1_hi = nullptr, *w1_lo = nullptr, *w2_hi = nullptr, *w2_lo = nullptr;
  void plan(Alloc& al, bool strict) {
    auto take = [&](size_t c) -> void* {
      return strict ? (void*)al.template take<float>(c) : (void*)al.template take<__nv_bfloat16>(c);
    };
    w1_hi = take(1024 * 128);
    if (strict) w1_lo = take(1024 * 128);
    w2_hi = take(128 * 512);
    if (strict) w2_lo = take(128 * 512);
  }
};

}  // namespace fpb

using namespace fpb;

extern "C" size_t fpb_transition_workspace_size(int c_z, int expansion, int precision) {
  if (c_z != 128 || expansion != 4 || (precision != 0 && precision != 1)) return 0;
  WsCounter cnt;
  TransPlan<WsCounter> pl;
  pl.plan(cnt, precision == 0);
  return cnt.used;
}

extern "C" int fpb_transition(float* z, float* delta_out, long long rows, int c_z, int expansion,
                              const float* ln_w, const float* ln_b, const float* w_a,
                              const float* w_b, const float* w_out, float eps, int precision,
                              void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!z || !ln_w || !ln_b || !w_a || !w_b || !w_out || !workspace) return kErrArg;
  if (delta_out && !aligned16(delta_out)) return kErrAlign;
  if (c_z != 128 || expansion != 4 || rows <= 0) return kErrShape;
  if (rows > 0x7fffffffll) return kErrShape;
  if (precision != 0 && precision != 1) return kErrArg;
  if (!aligned16(z) || !aligned16(workspace) || !aligned16(ln_w) || !aligned16(ln_b))
    return kErrAlign;
  if (workspace_bytes < fpb_transition_workspace_size(c_z, expansion, precision))
    return kErrWorkspace;
  const bool strict = precision == 0;
  WsCursor cur(workspace, workspace_bytes);
  TransPlan<WsCursor> pl;
  pl.plan(cur, strict);
  if (!cur.ok) return kErrWorkspace;
  if (reset_status(workspace, stream)) return kErrCuda;
  const int hc = strict ? TransCfg<true>::HC : TransCfg<false>::HC;
  FPB_LAUNCH("pack_weights", stream,
             pack_transition_w1<<<128, 256, 0, stream>>>(w_a, w_b, hc, pl.w1_hi, pl.w1_lo,
                                                         strict ? 1 : 0));
  FPB_LAUNCH("pack_weights", stream,
             pack_plain<<<64, 256, 0, stream>>>(w_out, 128 * 512, pl.w2_hi, pl.w2_lo,
                                                strict ? 1 : 0));
  int st;
  if ((st = launch_status())) return st;
  const int esz = strict ? 4 : 2;
  const CUtensorMapDataType dt =
      strict ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap m1h, m1l, m2h, m2l;
  bool ok = make_map_3d(&m1h, pl.w1_hi, dt, 128, 1024, 1, 128ull * esz, 128ull * esz * 1024,
                        128 / esz, 2 * hc, 1) &&
            make_map_3d(&m2h, pl.w2_hi, dt, 512, 128, 1, 512ull * esz, 512ull * esz * 128,
                        128 / esz, 128, 1);
  if (strict)
    ok = ok &&
         make_map_3d(&m1l, pl.w1_lo, dt, 128, 1024, 1, 128ull * esz, 128ull * esz * 1024,
                     128 / esz, 2 * hc, 1) &&
         make_map_3d(&m2l, pl.w2_lo, dt, 512, 128, 1, 512ull * esz, 512ull * esz * 128, 128 / esz,
                     128, 1);
  else {
    m1l = m1h;
    m2l = m2h;
  }
  if (!ok) return kErrArg;
  TransArgs ta{z, delta_out, (int)rows, eps, ln_w, ln_b, static_cast<int*>(workspace)};
  const unsigned tiles = (unsigned)((rows + 127) / 128);
  const unsigned grid = tiles < (unsigned)sm_count() ? tiles : (unsigned)sm_count();
  if (strict) {
    auto k = transition_kernel<true>;
    if (int smem_st = set_max_smem(k, TransCfg<true>::SMEM)) return smem_st;
    FPB_LAUNCH("transition", stream,
               k<<<grid, 192, TransCfg<true>::SMEM, stream>>>(m1h, m1l, m2h, m2l, ta));
  } else {
    auto k = transition_kernel<false>;
    if (int smem_st = set_max_smem(k, TransCfg<false>::SMEM)) return smem_st;
    FPB_LAUNCH("transition", stream,
               k<<<grid, 192, TransCfg<false>::SMEM, stream>>>(m1h, m1l, m2h, m2l, ta));
  }
  return launch_status();
}

// ============================================================================
// Allocation-free variant: the scratch lives in a static device array
// ============================================================================
// Same kernels and results as fpb_transition; the packed weights and the
// status word go to g_transition_scratch instead of a caller workspace, and
// the launches bypass the timing hook (which creates events when enabled).
namespace fpb {
namespace {

constexpr size_t kTransitionScratchBytes = FPB_TRANSITION_SCRATCH_BYTES;

// One instance per device. Every call overwrites the packed weights in full;
// only the 256-byte status header must start at zero, and each call zeroes
// it on its own stream before its first kernel.
static __device__ __align__(256) unsigned char g_transition_scratch[kTransitionScratchBytes];

// Device address of the array in the current device's current context. The
// name g_transition_scratch is a host-side stand-in in host code, so the
// address is looked up, and it is looked up on every call: a cached value
// would outlive a cudaDeviceReset or belong to another context made current
// on the same device. The lookup is a host-side query (no stream work); the
// first one on a device may load this library's device code there.
int transition_scratch(void** out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_transition_scratch) != cudaSuccess || p == nullptr) {
    cudaGetLastError();
    return kErrCuda;
  }
  *out = p;
  return kOk;
}

}  // namespace
}  // namespace fpb

extern "C" int fpb_transition_noalloc(float* z, float* delta_out, long long rows, int c_z,
                                      int expansion, const float* ln_w, const float* ln_b,
                                      const float* w_a, const float* w_b, const float* w_out,
                                      float eps, int precision, int* status_out,
                                      cudaStream_t stream) {
  if (!z || !ln_w || !ln_b || !w_a || !w_b || !w_out) return kErrArg;
  if (delta_out && !aligned16(delta_out)) return kErrAlign;
  if (c_z != 128 || expansion != 4 || rows <= 0 || rows > 0x7fffffffll) return kErrShape;
  if (precision != 0 && precision != 1) return kErrArg;
  if (!aligned16(z) || !aligned16(ln_w) || !aligned16(ln_b)) return kErrAlign;
  const size_t need = fpb_transition_workspace_size(c_z, expansion, precision);
  if (need == 0) return kErrShape;
  if (need > kTransitionScratchBytes) return kErrScratch;
  if (status_out) {
    // reporting the status waits for the stream, which a capture forbids
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
      cudaGetLastError();
      return kErrCuda;
    }
    if (cap != cudaStreamCaptureStatusNone) return kErrArg;
  }
  void* scratch = nullptr;
  int st = transition_scratch(&scratch);
  if (st) return st;
  const bool strict = precision == 0;
  WsCursor cur(scratch, kTransitionScratchBytes);
  TransPlan<WsCursor> pl;
  pl.plan(cur, strict);
  if (!cur.ok) return kErrScratch;
  if (cudaMemsetAsync(scratch, 0, kWsHeader, stream) != cudaSuccess) return kErrCuda;
  const int hc = strict ? TransCfg<true>::HC : TransCfg<false>::HC;
  pack_transition_w1<<<128, 256, 0, stream>>>(w_a, w_b, hc, pl.w1_hi, pl.w1_lo, strict ? 1 : 0);
  pack_plain<<<64, 256, 0, stream>>>(w_out, 128 * 512, pl.w2_hi, pl.w2_lo, strict ? 1 : 0);
  if ((st = launch_status())) return st;
  const int esz = strict ? 4 : 2;
  const CUtensorMapDataType dt =
      strict ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUtensorMap m1h, m1l, m2h, m2l;
  bool ok = make_map_3d(&m1h, pl.w1_hi, dt, 128, 1024, 1, 128ull * esz, 128ull * esz * 1024,
                        128 / esz, 2 * hc, 1) &&
            make_map_3d(&m2h, pl.w2_hi, dt, 512, 128, 1, 512ull * esz, 512ull * esz * 128,
                        128 / esz, 128, 1);
  if (strict)
    ok = ok &&
         make_map_3d(&m1l, pl.w1_lo, dt, 128, 1024, 1, 128ull * esz, 128ull * esz * 1024,
                     128 / esz, 2 * hc, 1) &&
         make_map_3d(&m2l, pl.w2_lo, dt, 512, 128, 1, 512ull * esz, 512ull * esz * 128, 128 / esz,
                     128, 1);
  else {
    m1l = m1h;
    m2l = m2h;
  }
  if (!ok) return kErrArg;
  TransArgs ta{z, delta_out, (int)rows, eps, ln_w, ln_b, static_cast<int*>(scratch)};
  const unsigned tiles = (unsigned)((rows + 127) / 128);
  const unsigned grid = tiles < (unsigned)sm_count() ? tiles : (unsigned)sm_count();
  if (strict) {
    auto k = transition_kernel<true>;
    if (int smem_st = set_max_smem(k, TransCfg<true>::SMEM)) return smem_st;
    k<<<grid, 192, TransCfg<true>::SMEM, stream>>>(m1h, m1l, m2h, m2l, ta);
  } else {
    auto k = transition_kernel<false>;
    if (int smem_st = set_max_smem(k, TransCfg<false>::SMEM)) return smem_st;
    k<<<grid, 192, TransCfg<false>::SMEM, stream>>>(m1h, m1l, m2h, m2l, ta);
  }
  if ((st = launch_status())) return st;
  if (status_out) {
    // wait for this call, then report its device status word
    int word = 0;
    if (cudaMemcpyAsync(&word, scratch, sizeof(int), cudaMemcpyDeviceToHost, stream) !=
            cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
      return kErrCuda;
    *status_out = word;
  }
  return kOk;
}
