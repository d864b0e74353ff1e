// Batched triangle contraction on tcgen05 tensor cores.
//
// For every channel c: X_c[i][j] = sum_k A_c[i][k] * B_c[j][k] (both operands
// K-major, i.e. "a @ b^T" per channel). This is the N^3 core of the triangle
// multiplicative update (outgoing form; the incoming form is fed with
// operands already laid out in transposed pair coordinates by the producer).
//
// Strict mode: 3xTF32 (hi*hi + hi*lo + lo*hi, fp32 accumulate in TMEM) from
// pre-split hi/lo operand arrays. Fast mode: BF16 operands, fp32 accumulate.
//
// CTA = 6 warps: warp 0 issues TMA loads, warp 1 owns TMEM and issues MMAs
// (one elected thread), warps 2-5 drain the 128x256 fp32 accumulator from
// TMEM and store it. Tile: 128 (i) x 256 (j), K streamed through a ring of
// shared-memory stages in 128-byte swizzled K-major atoms.
#include "kernels.h"

namespace fpb {

template <bool kStrict>
struct ContractCfg {
  static constexpr int BM = 128;
  static constexpr int BN_MAX = 256;
  static constexpr int KATOM = kStrict ? 32 : 64;  // elements per 128-byte row
  static constexpr int NSPLIT = kStrict ? 2 : 1;
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN_MAX * 128;     // room for the widest tile
  static constexpr int STAGE_BYTES = NSPLIT * (A_BYTES + B_BYTES);
  static constexpr int STAGES = kStrict ? 2 : 4;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(STAGES * STAGE_BYTES >= BM * 132 * 4, "owner epilogue staging fits the stages");
};

// Column tile: the widest of 256/192/128/64/32 that divides the B chunk
// (a tile never straddles two ranks' rows of an all-gather buffer).
inline int contract_bn(int chunk_rows, bool chunked) {
  if (!chunked) return 256;
  for (int bn : {256, 192, 128, 64, 32})
    if (chunk_rows % bn == 0) return bn;
  return 0;
}

__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

template <bool kStrict, class OutT>
__global__ void __launch_bounds__(192, 1)
    contract_kernel(const __grid_constant__ CUtensorMap ma_hi,
                    const __grid_constant__ CUtensorMap ma_lo,
                    const __grid_constant__ CUtensorMap mb_hi,
                    const __grid_constant__ CUtensorMap mb_lo, ContractArgs args) {
  using C = ContractCfg<kStrict>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* done = empty + C::STAGES;
  uint64_t* drain = done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int jt = blockIdx.x, it = blockIdx.y, ch = blockIdx.z;
  const int bn = args.bn;
  const uint32_t tmem_cols = bn <= 32 ? 32u : bn <= 64 ? 64u : bn <= 128 ? 128u : 256u;
  const int nk = (args.k + C::KATOM - 1) / C::KATOM;
  const int j0 = jt * bn;
  const int b_chunk = j0 / args.b_chunk_rows;
  const int b_row = j0 - b_chunk * args.b_chunk_rows;
  const uint32_t stage_tx = C::NSPLIT * (C::A_BYTES + bn * 128);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const Guard g{args.status, abort_flag};

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&ma_hi);
      tma_prefetch_desc(&mb_hi);
      if (kStrict) {
        tma_prefetch_desc(&ma_lo);
        tma_prefetch_desc(&mb_lo);
      }
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % C::STAGES;
        const uint32_t ph = (kb / C::STAGES) & 1;
        if (kb >= C::STAGES && !mbar_wait(&empty[s], ph ^ 1, g, 1)) break;
        uint8_t* st = smem + s * C::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], stage_tx);
        const int kx = kb * C::KATOM;
        tma_load_3d(st, &ma_hi, &full[s], kx, it * C::BM, ch);
        tma_load_4d(st + C::A_BYTES, &mb_hi, &full[s], kx, b_row, ch, b_chunk);
        if (kStrict) {
          tma_load_3d(st + C::A_BYTES + C::B_BYTES, &ma_lo, &full[s], kx, it * C::BM, ch);
          tma_load_4d(st + 2 * C::A_BYTES + C::B_BYTES, &mb_lo, &full[s], kx, b_row, ch, b_chunk);
        }
        ++issued;
      }
      if (g.aborted()) {
        // drain our own in-flight copies before the CTA releases its smem
        for (int kb = (issued > C::STAGES ? issued - C::STAGES : 0); kb < issued; ++kb)
          (void)mbar_wait(&full[kb % C::STAGES], (kb / C::STAGES) & 1, Guard{nullptr, abort_flag},
                          0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = kStrict ? idesc_tf32(C::BM, bn) : idesc_bf16(C::BM, bn);
      uint32_t acc = 0;
      bool ok = true;
      for (int kb = 0; kb < nk && ok; ++kb) {
        const int s = kb % C::STAGES;
        const uint32_t ph = (kb / C::STAGES) & 1;
        if (!mbar_wait(&full[s], ph, g, 2)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint8_t* st = smem + s * C::STAGE_BYTES;
        const uint32_t a_hi = smem_u32(st);
        const uint32_t b_hi = smem_u32(st + C::A_BYTES);
        const uint32_t a_lo = smem_u32(st + C::A_BYTES + C::B_BYTES);
        const uint32_t b_lo = smem_u32(st + 2 * C::A_BYTES + C::B_BYTES);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // 4 x 32-byte K steps per 128-byte atom
          const uint32_t off = kk * 32;
          const uint64_t dah = umma_desc_sw128(a_hi + off);
          const uint64_t dbh = umma_desc_sw128(b_hi + off);
          if (kStrict) {
            const uint64_t dal = umma_desc_sw128(a_lo + off);
            const uint64_t dbl = umma_desc_sw128(b_lo + off);
            umma_tf32(tmem, dah, dbh, idesc, acc);
            umma_tf32(tmem, dah, dbl, idesc, 1u);
            umma_tf32(tmem, dal, dbh, idesc, 1u);
          } else {
            umma_bf16(tmem, dah, dbh, idesc, acc);
          }
          acc = 1u;
        }
        umma_commit(&empty[s]);
      }
      if (ok) {
        umma_commit(done);
      } else {
        // let every issued MMA retire before TMEM/smem are released
        umma_commit(drain);
        (void)mbar_wait(drain, 0, Guard{nullptr, abort_flag}, 0);
      }
    }
  } else if (args.owners) {
    // owner epilogue (rows stored at the ranks that own them, over NVLink
    // for the other ranks): each 128-column block of the tile is staged in
    // the now idle stage memory, then every warp stores whole rows, 32
    // lanes x 16 bytes contiguous per instruction, so each remote write is
    // one 512-byte burst instead of 32 separate 16-byte pieces
    const int q = warp & 3;
    const bool waited = mbar_wait(done, 0, g, 3);
    if (!bar_any(!waited, 1, 128)) {
      tc_fence_after();
      constexpr int SP = 132;  // staged row pitch (floats): conflict-free 16-byte accesses
      float* stg = reinterpret_cast<float*>(smem);
      const int trow = q * 32 + lane;  // tile row drained from TMEM by this thread
      const int wq = warp - 2;         // this warp stores tile rows wq*32 .. wq*32+31
      const int cl = 4 * lane;         // this lane's 4 columns of a staged block
#pragma unroll 1
      for (int cb0 = 0; cb0 < bn; cb0 += 128) {
        const int w = min(128, bn - cb0);
#pragma unroll 1
        for (int c = 0; c < w; c += 32) {
          uint32_t r[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + cb0 + c, r);
          tmem_ld_wait();
#pragma unroll
          for (int v = 0; v < 8; ++v)
            *reinterpret_cast<float4*>(stg + trow * SP + c + 4 * v) =
                make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                            __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
        }
        named_sync(1, 128);
        const int col = j0 + cb0 + cl;
#pragma unroll 1
        for (int rr = 0; rr < 32; ++rr) {
          const int tr = wq * 32 + rr;
          const int row = it * C::BM + tr;
          if (row >= args.m) break;  // uniform across the warp
          if (cl >= w || col >= args.nn) continue;
          const int d = min(row / args.owner_rows, args.owners - 1);
          const size_t lr = (size_t)(row - d * args.owner_rows);
          OutT* out = reinterpret_cast<OutT*>(args.outs[d]) +
                      (((lr * args.njb + (col >> 7)) * 128 + ch + args.ch_off) << 7) +
                      (col & 127);
          const float4 v = *reinterpret_cast<const float4*>(stg + tr * SP + cl);
          if (col + 4 <= args.nn) {
            if constexpr (sizeof(OutT) == 4) {
              *reinterpret_cast<float4*>(out) = v;
            } else {
              __nv_bfloat162 h0 = __floats2bfloat162_rn(v.x, v.y);
              __nv_bfloat162 h1 = __floats2bfloat162_rn(v.z, v.w);
              *reinterpret_cast<uint2*>(out) =
                  make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
            }
          } else {
            const float e[4] = {v.x, v.y, v.z, v.w};
            for (int u = 0; u < 4 && col + u < args.nn; ++u) {
              if constexpr (sizeof(OutT) == 4)
                out[u] = e[u];
              else
                out[u] = __float2bfloat16_rn(e[u]);
            }
          }
        }
        named_sync(1, 128);  // the staged block is read before the next overwrites it
      }
    }
  } else {
    // epilogue: warps 2..5 -> TMEM lane quadrants (warp % 4)
    const int q = warp & 3;
    if (mbar_wait(done, 0, g, 3)) {
      tc_fence_after();
      const int row = it * C::BM + q * 32 + lane;
#pragma unroll 1
      for (int cb = 0; cb < bn / 32; ++cb) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + cb * 32, r);
        tmem_ld_wait();
        const int col0 = j0 + cb * 32;
        // `out` points at column 0 of this (channel, row) run, so that
        // out + col0 addresses columns col0..col0+31 in either layout
        OutT* out;
        if (args.owners) {
          const int d = min(row / args.owner_rows, args.owners - 1);
          const size_t lr = (size_t)(row - d * args.owner_rows);
          out = reinterpret_cast<OutT*>(args.outs[d]) +
                (((lr * args.njb + (col0 >> 7)) * 128 + ch + args.ch_off) << 7) + (col0 & 127) -
                col0;
        } else if (args.blocked)
          out = reinterpret_cast<OutT*>(args.out) +
                ((((size_t)row * args.njb + (col0 >> 7)) * (args.bchannels ? args.bchannels : 128) +
                   ch)
                 << 7) +
                (col0 & 127) - col0;
        else
          out = reinterpret_cast<OutT*>(args.out) + (size_t)ch * args.out_channel_stride +
                (size_t)row * args.ldo;
        if (row < args.m && col0 < args.nn) {
          const bool vec = (col0 + 32 <= args.nn) &&
                           ((reinterpret_cast<uintptr_t>(out + col0) & 15u) == 0u);
          if (vec) {
            if constexpr (sizeof(OutT) == 4) {
              float4* o4 = reinterpret_cast<float4*>(out + col0);
#pragma unroll
              for (int v = 0; v < 8; ++v)
                o4[v] = make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                    __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
            } else {
              uint4* o4 = reinterpret_cast<uint4*>(out + col0);
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(r[8 * v + 2 * e]),
                                                           __uint_as_float(r[8 * v + 2 * e + 1]));
                  w[e] = *reinterpret_cast<uint32_t*>(&h);
                }
                o4[v] = make_uint4(w[0], w[1], w[2], w[3]);
              }
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              if (col0 + e < args.nn) {
                const float v = __uint_as_float(r[e]);
                if constexpr (sizeof(OutT) == 4)
                  out[col0 + e] = v;
                else
                  out[col0 + e] = __float2bfloat16_rn(v);
              }
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

// ----------------------------------------------------------------------------
// host launcher
// ----------------------------------------------------------------------------
int launch_contract(const ContractOperands& op, const ContractArgs& args_in, cudaStream_t stream) {
  if (op.m <= 0 || op.nn <= 0 || op.k <= 0 || op.channels <= 0 || op.b_chunks <= 0 ||
      op.b_chunk_rows <= 0 || (long long)op.b_chunks * op.b_chunk_rows < op.nn)
    return kErrShape;
  const bool chunked = op.b_chunks > 1;
  const int bn = contract_bn(op.b_chunk_rows, chunked);
  if (bn == 0) return kErrShape;
  ContractArgs args = args_in;
  args.m = op.m;
  args.nn = op.nn;
  args.k = op.k;
  args.bn = bn;
  args.b_chunk_rows = op.b_chunk_rows;
  CUtensorMap mah{}, mal{}, mbh{}, mbl{};
  const bool strict = op.strict;
  const CUtensorMapDataType dt = strict ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                        : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int esz = strict ? 4 : 2;
  const int katom = 128 / esz;
  const uint64_t s1 = (uint64_t)op.ld * esz;
  const uint64_t sa2 = (uint64_t)op.a_channel_stride * esz;
  const uint64_t sb2 = (uint64_t)op.b_channel_stride * esz;
  const uint64_t sb3 = (uint64_t)op.b_chunk_stride * esz;
  if (s1 % 16 || sa2 % 16 || sb2 % 16 || (chunked && sb3 % 16)) return kErrAlign;
  // an unchunked B still uses the 4-D map with one chunk
  const uint64_t sb3m = chunked ? sb3 : sb2 * op.channels;
  bool ok = make_map_3d(&mah, op.a_hi, dt, op.k, op.m, op.channels, s1, sa2, katom, 128, 1) &&
            make_map_4d(&mbh, op.b_hi, dt, op.k, op.b_chunk_rows, op.channels, op.b_chunks, s1,
                        sb2, sb3m, katom, bn, 1, 1);
  if (strict)
    ok = ok && make_map_3d(&mal, op.a_lo, dt, op.k, op.m, op.channels, s1, sa2, katom, 128, 1) &&
         make_map_4d(&mbl, op.b_lo, dt, op.k, op.b_chunk_rows, op.channels, op.b_chunks, s1, sb2,
                     sb3m, katom, bn, 1, 1);
  else {
    mal = mah;
    mbl = mbh;
  }
  if (!ok) return kErrArg;
  dim3 grid((op.nn + bn - 1) / bn, (op.m + 127) / 128, op.channels);
  if (strict) {
    auto k = contract_kernel<true, float>;
    const int smem = ContractCfg<true>::SMEM_BYTES;
    if (int smem_st = set_max_smem(k, smem)) return smem_st;
    FPB_LAUNCH("contract_strict", stream, k<<<grid, 192, smem, stream>>>(mah, mal, mbh, mbl, args));
  } else {
    const int smem = ContractCfg<false>::SMEM_BYTES;
    if (args.out_bf16) {
      auto k = contract_kernel<false, __nv_bfloat16>;
      if (int smem_st = set_max_smem(k, smem)) return smem_st;
      FPB_LAUNCH("contract_fast", stream, k<<<grid, 192, smem, stream>>>(mah, mal, mbh, mbl, args));
    } else {
      auto k = contract_kernel<false, float>;
      if (int smem_st = set_max_smem(k, smem)) return smem_st;
      FPB_LAUNCH("contract_fast", stream, k<<<grid, 192, smem, stream>>>(mah, mal, mbh, mbl, args));
    }
  }
  return launch_status();
}

// ----------------------------------------------------------------------------
// operand preparation for the packed-BMM entry point: split (strict) or
// convert (fast) [batch][n][n] fp32 matrices into padded K-major operands,
// transposing them first for the incoming direction (a^T, b^T).
// ----------------------------------------------------------------------------
template <bool kStrict>
__global__ void prep_operand_kernel(const float* __restrict__ src, int n, int transpose,
                                    void* __restrict__ hi, void* __restrict__ lo, int ld,
                                    size_t channel_stride) {
  __shared__ float tile[32][33];
  const int ch = blockIdx.z;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const float* s = src + (size_t)ch * n * n;
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    const int r = r0 + y, c = c0 + threadIdx.x;
    tile[y][threadIdx.x] = (r < n && c < n) ? s[(size_t)r * n + c] : 0.f;
  }
  __syncthreads();
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    // output row/col (transposed when requested)
    const int orow = r0 + y, ocol = c0 + threadIdx.x;
    const float v = transpose ? tile[threadIdx.x][y] : tile[y][threadIdx.x];
    const int rr = transpose ? (c0 + y) : orow;
    const int cc = transpose ? (r0 + threadIdx.x) : ocol;
    if (rr < n && cc < n) {
      const size_t idx = (size_t)ch * channel_stride + (size_t)rr * ld + cc;
      if (kStrict) {
        float h, l;
        split_tf32(v, h, l);
        static_cast<float*>(hi)[idx] = h;
        static_cast<float*>(lo)[idx] = l;
      } else {
        static_cast<__nv_bfloat16*>(hi)[idx] = __float2bfloat16_rn(v);
      }
    }
  }
}

static void plan_packed_bmm(int batch, int n, int precision, WsCounter* cnt, WsCursor* cur,
                            void** a_hi, void** a_lo, void** b_hi, void** b_lo, int* ld,
                            size_t* cstride) {
  const bool strict = precision == 0;
  const int esz = strict ? 4 : 2;
  *ld = padded_ld(n, esz);
  *cstride = (size_t)n * (*ld);
  const size_t count = (size_t)batch * (*cstride);
  auto take = [&](void** p) {
    if (cur) {
      *p = strict ? (void*)cur->take<float>(count) : (void*)cur->take<__nv_bfloat16>(count);
    } else {
      if (strict)
        cnt->take<float>(count);
      else
        cnt->take<__nv_bfloat16>(count);
    }
  };
  take(a_hi);
  if (strict) take(a_lo);
  take(b_hi);
  if (strict) take(b_lo);
}

}  // namespace fpb

using namespace fpb;

extern "C" size_t fpb_packed_bmm_workspace_size(int batch, int n, int precision) {
  if (batch <= 0 || n <= 0) return 0;
  WsCounter cnt;
  void *a, *b, *c, *d;
  int ld;
  size_t cs;
  plan_packed_bmm(batch, n, precision, &cnt, nullptr, &a, &b, &c, &d, &ld, &cs);
  return cnt.used;
}

extern "C" int fpb_packed_bmm(const float* a, const float* b, float* out, int batch, int n,
                              int outgoing, int precision, void* workspace,
                              size_t workspace_bytes, cudaStream_t stream) {
  if (!a || !b || !out || !workspace) return kErrArg;
  if (batch <= 0 || n <= 0) return kErrShape;
  if (precision != 0 && precision != 1) return kErrArg;
  if (!aligned16(a) || !aligned16(b) || !aligned16(out) || !aligned16(workspace)) return kErrAlign;
  if (workspace_bytes < fpb_packed_bmm_workspace_size(batch, n, precision)) return kErrWorkspace;
  WsCursor cur(workspace, workspace_bytes);
  void *a_hi = nullptr, *a_lo = nullptr, *b_hi = nullptr, *b_lo = nullptr;
  int ld;
  size_t cs;
  plan_packed_bmm(batch, n, precision, nullptr, &cur, &a_hi, &a_lo, &b_hi, &b_lo, &ld, &cs);
  if (!cur.ok) return kErrWorkspace;
  const bool strict = precision == 0;
  // outgoing: X = A B^T (operands already K-major); incoming: X = A^T B, so
  // both operands are transposed into K-major form.
  const int tr = outgoing ? 0 : 1;
  dim3 pg((n + 31) / 32, (n + 31) / 32, batch), pb(32, 8);
  if (strict) {
    FPB_LAUNCH("prep_operand", stream,
               prep_operand_kernel<true><<<pg, pb, 0, stream>>>(a, n, tr, a_hi, a_lo, ld, cs));
    FPB_LAUNCH("prep_operand", stream,
               prep_operand_kernel<true><<<pg, pb, 0, stream>>>(b, n, tr, b_hi, b_lo, ld, cs));
  } else {
    FPB_LAUNCH("prep_operand", stream,
               prep_operand_kernel<false><<<pg, pb, 0, stream>>>(a, n, tr, a_hi, nullptr, ld, cs));
    FPB_LAUNCH("prep_operand", stream,
               prep_operand_kernel<false><<<pg, pb, 0, stream>>>(b, n, tr, b_hi, nullptr, ld, cs));
  }
  if (cudaGetLastError() != cudaSuccess) return kErrCuda;
  if (reset_status(workspace, stream)) return kErrCuda;
  ContractOperands op{a_hi, a_lo, b_hi, b_lo, ld, cs, cs, n, n, n, n, 1, 0, batch, strict};
  ContractArgs args{};
  args.out = out;
  args.ldo = n;
  args.out_channel_stride = (size_t)n * n;
  args.out_bf16 = 0;
  args.status = static_cast<int*>(workspace);
  return launch_contract(op, args, stream);
}
