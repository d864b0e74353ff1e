// Single stack of a Pairformer block on sm_100a: AttentionPairBias without
// conditioning (AlphaFold 3 Algorithm 24, as the upstream Protenix trunk
// runs it) and the single transition (Algorithm 11), each added to s.
//
//   a = LN(s);  q = a Wq^T + bq;  k, v, g = a Wk^T, a Wv^T, a Wg^T
//   b^h_ij = LN(z_ij) Wz^T + 1e9 (mask_ij - 1)              (16 heads)
//   s_i += W_o (sigmoid(g_i) * sum_j softmax_j(q_i.k_j / sqrt(24) + b_ij) v_j)
//   s_i += W_out(silu(LN(s_i) Wa^T) * (LN(s_i) Wb^T))
//
// The reference runs this stack natively (it is not accelerated there,
// docs/openfold3-performance.md:68-74). It is 0.3 % of the block's FLOPs
// (about 5.6e3 N^2 + 4.7e6 N), so it runs as FP32 CUDA-core kernels, exact to
// FP32 rounding in both precision modes. A call owns query rows
// [r0, r0 + rows) of s (all rows of s are read for k and v), so the
// row-sharded path runs it on each rank's rows and all-gathers s afterwards.
#include "../../include/fireprot_b200.h"
#include "kernels.h"
#include "rowgemm.cuh"

namespace fpb {

constexpr int kSHeads = 16;
constexpr int kSDim = 24;
constexpr int kCs = 384;
constexpr int kSHid = 4 * kCs;
constexpr float kSMaskInf = 1e9f;

// ---------------------------------------------------------------- LayerNorm
// one warp per row of c = 384 channels (12 per lane), biased variance
__global__ void ln_rows384_kernel(const float* __restrict__ x, float* __restrict__ y, int rows,
                                  const float* __restrict__ w, const float* __restrict__ b,
                                  float eps) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)warp * kCs);
  float4 v[3];
  float s = 0.f;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    v[u] = xr[u * 32 + lane];
    s += v[u].x + v[u].y + v[u].z + v[u].w;
  }
  const float mean = warp_sum(s) * (1.0f / kCs);
  float q = 0.f;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    const float d0 = v[u].x - mean, d1 = v[u].y - mean, d2 = v[u].z - mean, d3 = v[u].w - mean;
    q += d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3;
  }
  const float rs = rsqrtf(warp_sum(q) * (1.0f / kCs) + eps);
  float4* yr = reinterpret_cast<float4*>(y + (size_t)warp * kCs);
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    const int c = (u * 32 + lane) * 4;
    yr[u * 32 + lane] = make_float4((v[u].x - mean) * rs * w[c] + b[c],
                                    (v[u].y - mean) * rs * w[c + 1] + b[c + 1],
                                    (v[u].z - mean) * rs * w[c + 2] + b[c + 2],
                                    (v[u].w - mean) * rs * w[c + 3] + b[c + 3]);
  }
}

// ---------------------------------------------------------------- SGEMM
// C[M][N] (op)= A[M][K] W[N][K]^T in FP32: 64 x 64 tiles, K steps of 16,
// 256 threads with 4 x 4 outputs each. K is a multiple of 16 and every
// leading dimension a multiple of 4 (384 or 1536 here).
// kEpiHeads stores head-major: column h*24 + d of row m goes to
// Cm[(h * M + m) * 24 + d] (the attention's key / value layout).
enum SgemmEpi { kEpiStore = 0, kEpiBias = 1, kEpiSigmoid = 2, kEpiAdd = 3, kEpiHeads = 4 };

template <int kEpi>
__global__ void __launch_bounds__(256)
    sgemm_nt_kernel(const float* __restrict__ A, int lda, const float* __restrict__ W, int ldw,
                    float* __restrict__ Cm, int ldc, int M, int N, int K,
                    const float* __restrict__ bias) {
  __shared__ __align__(16) float As[16][64 + 4];
  __shared__ __align__(16) float Ws[16][64 + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  // loader: 256 threads x one float4 = 64 rows x 16 k of each operand
  const int lr = threadIdx.x >> 2, lk = (threadIdx.x & 3) * 4;
  for (int k0 = 0; k0 < K; k0 += 16) {
    const int am = m0 + lr, wn = n0 + lr;
    const float4 av = am < M ? *reinterpret_cast<const float4*>(A + (size_t)am * lda + k0 + lk)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 wv = wn < N ? *reinterpret_cast<const float4*>(W + (size_t)wn * ldw + k0 + lk)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
    As[lk][lr] = av.x;
    As[lk + 1][lr] = av.y;
    As[lk + 2][lr] = av.z;
    As[lk + 3][lr] = av.w;
    Ws[lk][lr] = wv.x;
    Ws[lk + 1][lr] = wv.y;
    Ws[lk + 2][lr] = wv.z;
    Ws[lk + 3][lr] = wv.w;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      const float4 a4 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 w4 = *reinterpret_cast<const float4*>(&Ws[kk][tx * 4]);
      const float av4[4] = {a4.x, a4.y, a4.z, a4.w};
      const float wv4[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[u][v] = fmaf(av4[u], wv4[v], acc[u][v]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int m = m0 + ty * 4 + u;
    if (m >= M) continue;
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int nn = n0 + tx * 4 + v;
      if (nn >= N) continue;
      float r = acc[u][v];
      float* dst = kEpi == kEpiHeads
                       ? Cm + ((size_t)(nn / kSDim) * M + m) * kSDim + nn % kSDim
                       : Cm + (size_t)m * ldc + nn;
      if constexpr (kEpi == kEpiBias) r += bias[nn];
      if constexpr (kEpi == kEpiSigmoid) r = sigmoidf_(r);
      if constexpr (kEpi == kEpiAdd) r += *dst;
      *dst = r;
    }
  }
}

template <int kEpi>
void sgemm_nt(const float* A, int lda, const float* W, int ldw, float* Cm, int ldc, int M, int N,
              int K, const float* bias, cudaStream_t stream) {
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  FPB_LAUNCH("single_gemm", stream,
             (sgemm_nt_kernel<kEpi><<<grid, 256, 0, stream>>>(A, lda, W, ldw, Cm, ldc, M, N, K,
                                                              bias)));
}

// ---------------------------------------------------------------- cp.async
// 16-byte global -> shared copies (no register staging); completion is the
// hardware group wait, not a spin loop.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

// ---------------------------------------------------------------- pair bias
// LayerNorm affine folded into the head weights, once per call:
//   wp[c][h] = ln_w[c] Wz[h][c],  bp[h] = sum_c ln_b[c] Wz[h][c]
// so that LN(z) Wz^T = rs * sum_c (z_c - mean) wp[c][h] + bp[h].
constexpr int kPBWeights = 128 * kSHeads + kSHeads;

__global__ void single_bias_weights_kernel(const float* __restrict__ ln_w,
                                           const float* __restrict__ ln_b,
                                           const float* __restrict__ wz, float* __restrict__ out) {
  __shared__ float part[4][kSHeads];
  const int c = threadIdx.x, lane = c & 31, warp = c >> 5;  // 128 threads = channels
#pragma unroll
  for (int h = 0; h < kSHeads; ++h) {
    const float w = wz[h * 128 + c];
    out[c * kSHeads + h] = ln_w[c] * w;
    const float t = warp_sum(ln_b[c] * w);
    if (lane == 0) part[warp][h] = t;
  }
  __syncthreads();
  if (c < kSHeads) out[128 * kSHeads + c] = part[0][c] + part[1][c] + part[2][c] + part[3][c];
}

// biasT[h][j][i - r0] = LN(z_ij) Wz^T + 1e9 (mask_ij - 1) for the call's query
// rows i. A block takes 128 query rows i of one key column j; warp w copies
// the pair rows of its own 32 queries (512 bytes each, one warp-wide
// 16-byte cp.async per row) into shared memory and waits for its own copies
// only, so the warps of a block overlap loading and computing. Lane l then
// normalises its row (two passes) and forms its 16 head values: every store
// is a 32-query coalesced segment of biasT.
constexpr int kPBRows = 128;
constexpr int kPBThreads = 2 * kPBRows;  // two threads per row, 8 heads each
constexpr int kPBStride = 132;  // floats per staged row: 16-byte aligned, no bank conflicts
constexpr int kPBSmem = (kPBRows * kPBStride + kPBWeights) * 4;

__global__ void __launch_bounds__(kPBThreads)
    single_pair_bias_kernel(const float* __restrict__ z_loc, const float* __restrict__ mask,
                            int n, int rows, int r0, const float* __restrict__ wfold, float eps,
                            float* __restrict__ biasT) {
  extern __shared__ float4 pb_smem4[];
  float* xs = reinterpret_cast<float*>(pb_smem4);
  float* wp = xs + kPBRows * kPBStride;
  const int iblocks = (rows + kPBRows - 1) / kPBRows;
  const int j = blockIdx.x / iblocks;
  const int i0 = (blockIdx.x % iblocks) * kPBRows;
  const int cnt = min(kPBRows, rows - i0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < kPBWeights; e += kPBThreads) wp[e] = wfold[e];
  // warp w stages rows [16 w, 16 w + 16), lane = 16-byte chunk of the row
  const int wr = max(0, min(16, cnt - warp * 16));
#pragma unroll 4
  for (int rr = 0; rr < wr; ++rr) {
    const int r = warp * 16 + rr;
    cp_async16(xs + r * kPBStride + lane * 4,
               z_loc + ((size_t)(i0 + r) * n + j) * 128 + lane * 4);
  }
  cp_async_commit();
  // thread (row, half): heads [8 half, 8 half + 8) of row `row`
  const int row = tid & (kPBRows - 1), half = tid / kPBRows;
  constexpr int kHalfHeads = kSHeads / 2;
  const int il = i0 + row;
  const float mb =
      (mask && row < cnt) ? kSMaskInf * (mask[(size_t)(r0 + il) * n + j] - 1.0f) : 0.f;
  cp_async_wait<0>();
  __syncthreads();  // rows staged by other warps; the weights
  if (row >= cnt) return;
  const float4* xr = reinterpret_cast<const float4*>(xs + row * kPBStride);
  float sum = 0.f;
#pragma unroll 8
  for (int c4 = 0; c4 < 32; ++c4) {
    const float4 x = xr[c4];
    sum += (x.x + x.y) + (x.z + x.w);
  }
  const float mean = sum * (1.0f / 128.0f);
  float acc[kHalfHeads];
#pragma unroll
  for (int h = 0; h < kHalfHeads; ++h) acc[h] = 0.f;
  float var = 0.f;
  const float4* w4 = reinterpret_cast<const float4*>(wp);
#pragma unroll 2
  for (int c4 = 0; c4 < 32; ++c4) {
    const float4 x = xr[c4];
    const float xc[4] = {x.x - mean, x.y - mean, x.z - mean, x.w - mean};
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      var = fmaf(xc[u], xc[u], var);
#pragma unroll
      for (int hq = 0; hq < kHalfHeads / 4; ++hq) {
        const float4 w = w4[(c4 * 4 + u) * (kSHeads / 4) + half * (kHalfHeads / 4) + hq];
        acc[hq * 4 + 0] = fmaf(xc[u], w.x, acc[hq * 4 + 0]);
        acc[hq * 4 + 1] = fmaf(xc[u], w.y, acc[hq * 4 + 1]);
        acc[hq * 4 + 2] = fmaf(xc[u], w.z, acc[hq * 4 + 2]);
        acc[hq * 4 + 3] = fmaf(xc[u], w.w, acc[hq * 4 + 3]);
      }
    }
  }
  const float rs = rsqrtf(var * (1.0f / 128.0f) + eps);
  const float* bp = wp + 128 * kSHeads;
#pragma unroll
  for (int hh = 0; hh < kHalfHeads; ++hh) {
    const int h = half * kHalfHeads + hh;
    biasT[((size_t)h * n + j) * rows + il] = fmaf(rs, acc[hh], bp[h]) + mb;
  }
}

// ---------------------------------------------------------------- attention
// o[i][h*24 + d] for the call's query rows. A block takes 32 queries (one
// per lane) of one head; its 4 warps split every 64-key tile (16 keys each)
// and keep their own online-softmax state, merged through shared memory at
// the end. k and v are head-major ([16][n][24]), so a tile of one head is one
// contiguous 6 KB block per operand, double-buffered by cp.async; the pair
// bias of the next tile is loaded into registers while the current one runs.
constexpr int kSAttnQ = 32;
constexpr int kSAttnWarps = 4;
constexpr int kSAttnTile = 64;
constexpr int kSAttnKW = kSAttnTile / kSAttnWarps;  // keys per warp per tile
constexpr int kSAttnTileF = kSAttnTile * kSDim;      // floats per operand tile

__device__ __forceinline__ void single_attn_load_tile(float* dst_k, float* dst_v,
                                                      const float* kg, const float* vg, int j0,
                                                      int n) {
  const int chunks = min(kSAttnTile, n - j0) * (kSDim / 4);  // 16-byte chunks per operand
  for (int e = threadIdx.x; e < chunks; e += kSAttnQ * kSAttnWarps) {
    cp_async16(dst_k + e * 4, kg + (size_t)j0 * kSDim + e * 4);
    cp_async16(dst_v + e * 4, vg + (size_t)j0 * kSDim + e * 4);
  }
}

__global__ void __launch_bounds__(kSAttnQ * kSAttnWarps, 3)
    single_attn_kernel(const float* __restrict__ q, const float* __restrict__ kh,
                       const float* __restrict__ vh, const float* __restrict__ biasT, int n,
                       int rows, float* __restrict__ o) {
  __shared__ __align__(16) float kv[2][2][kSAttnTileF];  // [buffer][k | v][key][24]
  const int h = blockIdx.y;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int il = blockIdx.x * kSAttnQ + lane;
  const bool valid = il < rows;
  const float* kg = kh + (size_t)h * n * kSDim;
  const float* vg = vh + (size_t)h * n * kSDim;
  const float* bg = biasT + (size_t)h * n * rows + (valid ? il : 0);
  const float scale = rsqrtf((float)kSDim);
  float qv[kSDim], ov[kSDim];
#pragma unroll
  for (int d = 0; d < kSDim; ++d) {
    qv[d] = valid ? q[(size_t)il * kCs + h * kSDim + d] * scale : 0.f;
    ov[d] = 0.f;
  }
  float m_run = -INFINITY, l_run = 0.f;
  const int ntiles = (n + kSAttnTile - 1) / kSAttnTile;
  single_attn_load_tile(kv[0][0], kv[0][1], kg, vg, 0, n);
  cp_async_commit();
  float bnext[kSAttnKW];
#pragma unroll
  for (int jj = 0; jj < kSAttnKW; ++jj) {
    const int j = warp * kSAttnKW + jj;
    bnext[jj] = (j < n && valid) ? bg[(size_t)j * rows] : 0.f;
  }
  for (int t = 0; t < ntiles; ++t) {
    const int buf = t & 1;
    if (t + 1 < ntiles) {
      single_attn_load_tile(kv[buf ^ 1][0], kv[buf ^ 1][1], kg, vg, (t + 1) * kSAttnTile, n);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int jw = t * kSAttnTile + warp * kSAttnKW;  // first key of this warp's slice
    float sc[kSAttnKW];
    float mx = -INFINITY;
    const float4* k4 = reinterpret_cast<const float4*>(kv[buf][0] + warp * kSAttnKW * kSDim);
#pragma unroll
    for (int jj = 0; jj < kSAttnKW; ++jj) {
      float s = -INFINITY;
      if (jw + jj < n) {
        float p0 = bnext[jj], p1 = 0.f;
#pragma unroll
        for (int d4 = 0; d4 < kSDim / 4; ++d4) {
          const float4 kk = k4[jj * (kSDim / 4) + d4];
          p0 = fmaf(qv[d4 * 4 + 0], kk.x, p0);
          p1 = fmaf(qv[d4 * 4 + 1], kk.y, p1);
          p0 = fmaf(qv[d4 * 4 + 2], kk.z, p0);
          p1 = fmaf(qv[d4 * 4 + 3], kk.w, p1);
        }
        s = p0 + p1;
      }
      sc[jj] = s;
      mx = fmaxf(mx, s);
    }
    // bias of the next tile: in flight while this tile's P V runs
    if (t + 1 < ntiles) {
#pragma unroll
      for (int jj = 0; jj < kSAttnKW; ++jj) {
        const int j = jw + kSAttnTile + jj;
        bnext[jj] = (j < n && valid) ? bg[(size_t)j * rows] : 0.f;
      }
    }
    const float m_new = fmaxf(m_run, mx);
    if (m_new != -INFINITY) {  // uniform: -inf only while no key of the slice is < n
      const float alpha = __expf(m_run - m_new);
      const float4* v4 = reinterpret_cast<const float4*>(kv[buf][1] + warp * kSAttnKW * kSDim);
      float ls = 0.f;
#pragma unroll
      for (int d = 0; d < kSDim; ++d) ov[d] *= alpha;
#pragma unroll
      for (int jj = 0; jj < kSAttnKW; ++jj) {
        if (jw + jj < n) {
          const float pj = __expf(sc[jj] - m_new);
          ls += pj;
#pragma unroll
          for (int d4 = 0; d4 < kSDim / 4; ++d4) {
            const float4 vv = v4[jj * (kSDim / 4) + d4];
            ov[d4 * 4 + 0] = fmaf(pj, vv.x, ov[d4 * 4 + 0]);
            ov[d4 * 4 + 1] = fmaf(pj, vv.y, ov[d4 * 4 + 1]);
            ov[d4 * 4 + 2] = fmaf(pj, vv.z, ov[d4 * 4 + 2]);
            ov[d4 * 4 + 3] = fmaf(pj, vv.w, ov[d4 * 4 + 3]);
          }
        }
      }
      l_run = l_run * alpha + ls;
      m_run = m_new;
    }
    __syncthreads();  // the buffer is refilled by the next iteration's copy
  }
  // merge the 4 key splits: state [warp][lane] = (m, l, o[24]) in the k/v space
  float* st = &kv[0][0][0];
  constexpr int kStateF = kSDim + 2;
  float* mine = st + (warp * kSAttnQ + lane) * kStateF;
  mine[0] = m_run;
  mine[1] = l_run;
#pragma unroll
  for (int d = 0; d < kSDim; ++d) mine[2 + d] = ov[d];
  __syncthreads();
  if (!valid) return;
  float mw[kSAttnWarps], M = -INFINITY;
#pragma unroll
  for (int w = 0; w < kSAttnWarps; ++w) {
    mw[w] = st[(w * kSAttnQ + lane) * kStateF];
    M = fmaxf(M, mw[w]);  // finite: warp 0 always holds key 0
  }
  float den = 0.f, sw[kSAttnWarps];
#pragma unroll
  for (int w = 0; w < kSAttnWarps; ++w) {
    sw[w] = __expf(mw[w] - M);  // 0 for a split that saw no key
    den = fmaf(sw[w], st[(w * kSAttnQ + lane) * kStateF + 1], den);
  }
  const float inv = 1.0f / den;
  // warp w writes dims [6w, 6w + 6) of its query
  constexpr int kDW = kSDim / kSAttnWarps;
#pragma unroll
  for (int u = 0; u < kDW; ++u) {
    const int d = warp * kDW + u;
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < kSAttnWarps; ++w)
      acc = fmaf(sw[w], st[(w * kSAttnQ + lane) * kStateF + 2 + d], acc);
    o[(size_t)il * kCs + h * kSDim + d] = acc * inv;
  }
}

// go = g * o (sigmoid already applied to g); h = silu(a) * b
__global__ void single_mul_kernel(const float* __restrict__ g, float* __restrict__ o,
                                  size_t count) {
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < count;
       e += (size_t)gridDim.x * blockDim.x)
    o[e] = g[e] * o[e];
}
__global__ void single_swiglu_kernel(float* __restrict__ a, const float* __restrict__ b,
                                     size_t count) {
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < count;
       e += (size_t)gridDim.x * blockDim.x) {
    const float x = a[e];
    a[e] = x * sigmoidf_(x) * b[e];
  }
}

template <class Alloc>
struct SinglePlan {
  float *a = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *g = nullptr, *o = nullptr;
  float *biasT = nullptr, *ta = nullptr, *tb = nullptr, *wfold = nullptr;
  void plan(Alloc& al, int n, int rows) {
    wfold = al.template take<float>(kPBWeights);
    a = al.template take<float>((size_t)n * kCs);  // LN(s), all rows
    q = al.template take<float>((size_t)rows * kCs);
    k = al.template take<float>((size_t)n * kCs);  // head-major [16][n][24]
    v = al.template take<float>((size_t)n * kCs);
    g = al.template take<float>((size_t)rows * kCs);
    o = al.template take<float>((size_t)rows * kCs);
    biasT = al.template take<float>((size_t)kSHeads * n * rows);
    ta = al.template take<float>((size_t)rows * kSHid);
    tb = al.template take<float>((size_t)rows * kSHid);
  }
};

unsigned grid_for(size_t count) {
  const size_t blocks = (count + 255) / 256;
  return (unsigned)(blocks < 8192 ? blocks : 8192);
}

}  // namespace fpb

using namespace fpb;

extern "C" size_t fpb_single_block_workspace_size(int n, int rows, int c_s) {
  if (n <= 0 || rows <= 0 || rows > n || c_s != kCs) return 0;
  WsCounter cnt;
  SinglePlan<WsCounter> pl;
  pl.plan(cnt, n, rows);
  return cnt.used;
}

extern "C" int fpb_single_block(float* s, const float* z_loc, const float* mask, int n, int rows,
                                int r0, int c_s, const fpb_single_block_weights* w, float eps,
                                int precision, void* workspace, size_t workspace_bytes,
                                cudaStream_t stream) {
  if (!s || !z_loc || !w || !workspace) return kErrArg;
  if (precision != 0 && precision != 1) return kErrArg;
  if (c_s != kCs || n <= 0 || rows <= 0 || r0 < 0 || (long long)r0 + rows > n)
    return kErrShape;
  if ((long long)kSHeads * n * rows > 0x7fffffffll * 8) return kErrShape;
  const float* need[] = {w->ln_a_w, w->ln_a_b, w->w_q,    w->b_q,    w->w_k,    w->w_v,
                         w->w_g,    w->w_o,    w->ln_z_w, w->ln_z_b, w->w_z,    w->tr_ln_w,
                         w->tr_ln_b, w->tr_w_a, w->tr_w_b, w->tr_w_out};
  for (const float* ptr : need)
    if (!ptr) return kErrArg;
  const void* vec[] = {s, z_loc, workspace, w->ln_z_w, w->ln_z_b, w->w_z, w->w_q, w->w_k,
                       w->w_v, w->w_g, w->w_o, w->tr_w_a, w->tr_w_b, w->tr_w_out};
  for (const void* ptr : vec)
    if (!aligned16(ptr)) return kErrAlign;
  if (workspace_bytes < fpb_single_block_workspace_size(n, rows, c_s)) return kErrWorkspace;
  WsCursor cur(workspace, workspace_bytes);
  SinglePlan<WsCursor> pl;
  pl.plan(cur, n, rows);
  if (!cur.ok) return kErrWorkspace;
  if (reset_status(workspace, stream)) return kErrCuda;
  float* s_mine = s + (size_t)r0 * kCs;
  const float* a_mine = pl.a + (size_t)r0 * kCs;
  // ---- attention with pair bias: k and v from every row of s; q, g and the
  // update on the call's rows. Every read of s precedes the first write.
  FPB_LAUNCH("single_ln", stream,
             (ln_rows384_kernel<<<(n + 7) / 8, 256, 0, stream>>>(s, pl.a, n, w->ln_a_w,
                                                                 w->ln_a_b, eps)));
  sgemm_nt<kEpiBias>(a_mine, kCs, w->w_q, kCs, pl.q, kCs, rows, kCs, kCs, w->b_q, stream);
  sgemm_nt<kEpiHeads>(pl.a, kCs, w->w_k, kCs, pl.k, kCs, n, kCs, kCs, nullptr, stream);
  sgemm_nt<kEpiHeads>(pl.a, kCs, w->w_v, kCs, pl.v, kCs, n, kCs, kCs, nullptr, stream);
  sgemm_nt<kEpiSigmoid>(a_mine, kCs, w->w_g, kCs, pl.g, kCs, rows, kCs, kCs, nullptr, stream);
  FPB_LAUNCH("single_bias_weights", stream,
             (single_bias_weights_kernel<<<1, 128, 0, stream>>>(w->ln_z_w, w->ln_z_b, w->w_z,
                                                                pl.wfold)));
  {
    const long long blocks = (long long)n * ((rows + kPBRows - 1) / kPBRows);
    if (blocks > 0x7fffffffll) return kErrShape;
    if (int smem_st = set_max_smem(single_pair_bias_kernel, kPBSmem)) return smem_st;
    FPB_LAUNCH("single_pair_bias", stream,
               (single_pair_bias_kernel<<<(unsigned)blocks, kPBThreads, kPBSmem, stream>>>(
                   z_loc, mask, n, rows, r0, pl.wfold, eps, pl.biasT)));
  }
  FPB_LAUNCH("single_attn", stream,
             (single_attn_kernel<<<dim3((rows + kSAttnQ - 1) / kSAttnQ, kSHeads),
                                   kSAttnQ * kSAttnWarps, 0, stream>>>(pl.q, pl.k, pl.v,
                                                                       pl.biasT, n, rows, pl.o)));
  const size_t cnt = (size_t)rows * kCs;
  FPB_LAUNCH("single_elementwise", stream,
             (single_mul_kernel<<<grid_for(cnt), 256, 0, stream>>>(pl.g, pl.o, cnt)));
  sgemm_nt<kEpiAdd>(pl.o, kCs, w->w_o, kCs, s_mine, kCs, rows, kCs, kCs, nullptr, stream);
  // ---- single transition on the call's rows (LN(s) reuses the q buffer)
  FPB_LAUNCH("single_ln", stream,
             (ln_rows384_kernel<<<(rows + 7) / 8, 256, 0, stream>>>(s_mine, pl.q, rows,
                                                                    w->tr_ln_w, w->tr_ln_b,
                                                                    eps)));
  sgemm_nt<kEpiStore>(pl.q, kCs, w->tr_w_a, kCs, pl.ta, kSHid, rows, kSHid, kCs, nullptr, stream);
  sgemm_nt<kEpiStore>(pl.q, kCs, w->tr_w_b, kCs, pl.tb, kSHid, rows, kSHid, kCs, nullptr, stream);
  const size_t hc = (size_t)rows * kSHid;
  FPB_LAUNCH("single_elementwise", stream,
             (single_swiglu_kernel<<<grid_for(hc), 256, 0, stream>>>(pl.ta, pl.tb, hc)));
  sgemm_nt<kEpiAdd>(pl.ta, kSHid, w->tr_w_out, kSHid, s_mine, kCs, rows, kCs, kSHid, nullptr,
                    stream);
  return launch_status();
}
