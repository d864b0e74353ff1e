// Pair-row GEMM building blocks: a tile of 128 pair rows (c = 128 channels
// each) times a small weight matrix, on tcgen05 tensor cores.
//
//  - The A operand (128 rows x K=128) is produced in shared memory by the
//    CTA's row warps (LayerNorm or another prologue), in the K-major 128-byte
//    swizzled layout the UMMA descriptors expect; strict mode stores it as a
//    tf32 hi/lo pair, fast mode as BF16.
//  - Weights [Nout][128] (pre-split hi/lo, or BF16) stream through a ring of
//    shared-memory stages via TMA, one [128 rows x 128 bytes] K-atom per
//    stage.
//  - Accumulators live in TMEM; row t of the tile is TMEM lane t, so the
//    epilogue thread that owns row t reads its outputs with tcgen05.ld.
#pragma once

#include "sm100.cuh"

namespace fpb {

template <bool kStrict>
struct RowCfg {
  static constexpr int ESZ = kStrict ? 4 : 2;
  static constexpr int KATOM = 128 / ESZ;            // elements per 128-byte atom row
  static constexpr int NKA = 128 / KATOM;            // K atoms for K = 128 (4 or 2)
  static constexpr int ATOM_BYTES = 128 * 128;       // 128 rows x 128 bytes
  static constexpr int NSPLIT = kStrict ? 2 : 1;
  static constexpr int A_SPLIT_BYTES = NKA * ATOM_BYTES;     // one split of A (64K / 32K)
  static constexpr int A_BYTES = NSPLIT * A_SPLIT_BYTES;     // 128K strict, 32K fast
  static constexpr int WSTAGE_BYTES = NSPLIT * ATOM_BYTES;   // 32K strict, 16K fast
};

// ---------------------------------------------------------------------------
// A-operand writers
// ---------------------------------------------------------------------------
// Lane-cooperative write of 4 consecutive channels (c0..c0+3) of `row`.
template <bool kStrict>
__device__ __forceinline__ void a_store4(uint8_t* a_base, int row, int c0, float v0, float v1,
                                         float v2, float v3) {
  using C = RowCfg<kStrict>;
  const int atom = c0 / C::KATOM;
  const int byte = (c0 % C::KATOM) * C::ESZ;
  uint8_t* p = a_base + atom * C::ATOM_BYTES + sw128_offset(row, byte);
  if constexpr (kStrict) {
    float h0, l0, h1, l1, h2, l2, h3, l3;
    split_tf32(v0, h0, l0);
    split_tf32(v1, h1, l1);
    split_tf32(v2, h2, l2);
    split_tf32(v3, h3, l3);
    *reinterpret_cast<float4*>(p) = make_float4(h0, h1, h2, h3);
    *reinterpret_cast<float4*>(p + C::A_SPLIT_BYTES) = make_float4(l0, l1, l2, l3);
  } else {
    __nv_bfloat162 a = __floats2bfloat162_rn(v0, v1);
    __nv_bfloat162 b = __floats2bfloat162_rn(v2, v3);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&a);
    w.y = *reinterpret_cast<uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = w;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Two-pass LayerNorm of one 128-channel row held as float4 by the 32 lanes
// of a warp (lane l owns channels 4l..4l+3); biased variance, eps inside the
// square root, as torch's layer_norm.
__device__ __forceinline__ float4 ln_row_warp(float4 x, float4 w, float4 b, float eps) {
  const float mean = warp_sum(x.x + x.y + x.z + x.w) * (1.0f / 128.0f);
  const float d0 = x.x - mean, d1 = x.y - mean, d2 = x.z - mean, d3 = x.w - mean;
  const float var = warp_sum(d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3) * (1.0f / 128.0f);
  const float rs = rsqrtf(var + eps);
  return make_float4(d0 * rs * w.x + b.x, d1 * rs * w.y + b.y, d2 * rs * w.z + b.z,
                     d3 * rs * w.w + b.w);
}

// LayerNorm of the kRows pair rows [row0, row0 + kRows) of a tile into the
// A operand, warp-cooperative (lane l owns channels 4l..4l+3). `src(row)`
// returns the row's float4 base pointer, or nullptr for a padding row
// (normalised from zeros). Every load of a batch of kBatch rows is issued
// before the batch's first row is normalised, so a warp pays kRows / kBatch
// memory round trips per tile. `per_row(row, y)` sees each normalised row
// (called by the whole warp). kNC: the rows are not written during the
// kernel by anyone but this CTA, after this call (non-coherent loads).
template <bool kStrict, int kBatch, bool kNC, class Src, class PerRow, int kRows = 32>
__device__ __forceinline__ void ln_rows_to_a(uint8_t* A, int row0, const Src& src, float4 lw,
                                             float4 lb, float eps, const PerRow& per_row) {
  static_assert(kRows % kBatch == 0, "batch must divide the warp's rows");
  const int lane = threadIdx.x & 31;
#pragma unroll 1
  for (int b0 = 0; b0 < kRows; b0 += kBatch) {
    float4 x[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const float4* ptr = src(row0 + b0 + u);
      x[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ptr) x[u] = kNC ? __ldg(ptr + lane) : ptr[lane];
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const float4 y = ln_row_warp(x[u], lw, lb, eps);
      a_store4<kStrict>(A, row0 + b0 + u, lane * 4, y.x, y.y, y.z, y.w);
      per_row(row0 + b0 + u, y);
    }
  }
}

// Strict-mode LayerNorm of the kRows rows [row0, row0 + kRows) from raw
// FP32 rows already in shared memory: the tile's z rows were copied by TMA
// (128-byte swizzle, one box per 32-channel K atom) into the lo half of A,
// exactly where lo(row, c) belongs. Lane l reads channels 4l..4l+3 of a row,
// normalises, and writes hi and lo over the same positions (each lane
// overwrites only what it read). `per_row(row, y)` as in ln_rows_to_a.
template <int kRows, class PerRow>
__device__ __forceinline__ void ln_smem_rows_to_a(uint8_t* A, int row0, float4 lw, float4 lb,
                                                  float eps, const PerRow& per_row) {
  using C = RowCfg<true>;
  constexpr int kBatch = 8;  // rows normalised together (independent reductions)
  static_assert(kRows % kBatch == 0, "batch must divide the rows");
  const int lane = threadIdx.x & 31;
  const int atom = lane / 8, byte = (lane % 8) * 16;
  const uint8_t* raw = A + C::A_SPLIT_BYTES + atom * C::ATOM_BYTES;
#pragma unroll 1
  for (int b0 = 0; b0 < kRows; b0 += kBatch) {
    float4 x[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      x[u] = *reinterpret_cast<const float4*>(raw + sw128_offset(row0 + b0 + u, byte));
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const float4 y = ln_row_warp(x[u], lw, lb, eps);
      a_store4<true>(A, row0 + b0 + u, lane * 4, y.x, y.y, y.z, y.w);
      per_row(row0 + b0 + u, y);
    }
  }
}

// Strict-mode A operand from raw FP32 rows already in shared memory (copied
// by TMA into the lo half of A, as for ln_smem_rows_to_a): the kRows rows
// [row0, row0 + kRows) are split in place into tf32 hi and lo, no other
// arithmetic. Lane l handles channels 4l..4l+3 of each row.
template <int kRows>
__device__ __forceinline__ void split_smem_rows_to_a(uint8_t* A, int row0) {
  using C = RowCfg<true>;
  constexpr int kBatch = 8;
  static_assert(kRows % kBatch == 0, "batch must divide the rows");
  const int lane = threadIdx.x & 31;
  const int atom = lane / 8, byte = (lane % 8) * 16;
  const uint8_t* raw = A + C::A_SPLIT_BYTES + atom * C::ATOM_BYTES;
#pragma unroll 1
  for (int b0 = 0; b0 < kRows; b0 += kBatch) {
    float4 x[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      x[u] = *reinterpret_cast<const float4*>(raw + sw128_offset(row0 + b0 + u, byte));
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      a_store4<true>(A, row0 + b0 + u, lane * 4, x[u].x, x[u].y, x[u].z, x[u].w);
  }
}

struct NoRowHook {
  __device__ __forceinline__ void operator()(int, float4) const {}
};

// ---------------------------------------------------------------------------
// MMA issue for one K atom: D (+)= A[atom] x W_stage^T, N = n_cols.
// ---------------------------------------------------------------------------
template <bool kStrict>
__device__ __forceinline__ void mma_k_atom(uint32_t d_tmem, uint32_t a_hi, uint32_t a_lo,
                                           uint32_t w_hi, uint32_t w_lo, uint32_t idesc,
                                           bool first) {
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    const uint32_t off = kk * 32;
    const uint64_t dah = umma_desc_sw128(a_hi + off);
    const uint64_t dwh = umma_desc_sw128(w_hi + off);
    const uint32_t acc = (first && kk == 0) ? 0u : 1u;
    if constexpr (kStrict) {
      const uint64_t dal = umma_desc_sw128(a_lo + off);
      const uint64_t dwl = umma_desc_sw128(w_lo + off);
      umma_tf32(d_tmem, dah, dwh, idesc, acc);
      umma_tf32(d_tmem, dah, dwl, idesc, 1u);
      umma_tf32(d_tmem, dal, dwh, idesc, 1u);
    } else {
      umma_bf16(d_tmem, dah, dwh, idesc, acc);
    }
  }
}

// Ring of weight stages fed by TMA. The producer and the MMA thread walk the
// same sequence of loads; `seq` counts loads issued / consumed.
struct WRing {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  int stages;
  int stage_bytes;
};

template <bool kStrict>
__device__ __forceinline__ bool wring_push(const WRing& r, int seq, const CUtensorMap* m_hi,
                                           const CUtensorMap* m_lo, int kx, int row,
                                           const Guard& g) {
  const int s = seq % r.stages;
  const uint32_t ph = (seq / r.stages) & 1;
  if (seq >= r.stages && !mbar_wait(&r.empty[s], ph ^ 1, g, 11)) return false;
  uint8_t* st = r.base + s * r.stage_bytes;
  mbar_arrive_expect_tx(&r.full[s], RowCfg<kStrict>::WSTAGE_BYTES);
  tma_load_3d(st, m_hi, &r.full[s], kx, row, 0);
  if constexpr (kStrict) tma_load_3d(st + RowCfg<kStrict>::ATOM_BYTES, m_lo, &r.full[s], kx, row, 0);
  return true;
}

// Wait for stage `seq`; returns its smem address (hi) or 0 on abort.
__device__ __forceinline__ uint32_t wring_wait(const WRing& r, int seq, const Guard& g) {
  const int s = seq % r.stages;
  const uint32_t ph = (seq / r.stages) & 1;
  if (!mbar_wait(&r.full[s], ph, g, 12)) return 0;
  tc_fence_after();
  return smem_u32(r.base + s * r.stage_bytes);
}

__device__ __forceinline__ void wring_release(const WRing& r, int seq) {
  umma_commit(&r.empty[seq % r.stages]);
}

// Drain helper for the producer on abort: wait (bounded) for the last loads.
__device__ __forceinline__ void wring_drain(const WRing& r, int issued, volatile int* abort_flag) {
  for (int q = (issued > r.stages ? issued - r.stages : 0); q < issued; ++q)
    (void)mbar_wait(&r.full[q % r.stages], (q / r.stages) & 1, Guard{nullptr, abort_flag}, 0);
}

// TMEM row load helper: 32 consecutive fp32 columns of this thread's lane.
__device__ __forceinline__ void tmem_row32(uint32_t tmem_base, int quadrant, int col,
                                           float (&v)[32]) {
  uint32_t r[32];
  tmem_ld32(tmem_base + ((uint32_t)(quadrant * 32) << 16) + (uint32_t)col, r);
  tmem_ld_wait();
#pragma unroll
  for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
}

}  // namespace fpb
