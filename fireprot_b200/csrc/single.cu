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
enum SgemmEpi { kEpiStore = 0, kEpiBias = 1, kEpiSigmoid = 2, kEpiAdd = 3 };

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
      float* dst = Cm + (size_t)m * ldc + nn;
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

// ---------------------------------------------------------------- pair bias
// biasT[h][j][i - r0] = LN(z_ij) Wz^T + 1e9 (mask_ij - 1) for the call's query
// rows i. One warp per (key j, 32 query rows): each pair row is a coalesced
// 512-byte load, and lane l keeps the 16 head values of query i0 + l, so the
// stores are 128-byte rows.
__global__ void single_pair_bias_kernel(const float* __restrict__ z_loc,
                                        const float* __restrict__ mask, int n, int rows, int r0,
                                        const float* __restrict__ ln_w,
                                        const float* __restrict__ ln_b,
                                        const float* __restrict__ wz, float eps,
                                        float* __restrict__ biasT) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int iblocks = (rows + 31) / 32;
  if (warp >= n * iblocks) return;
  const int j = warp / iblocks, i0 = (warp % iblocks) * 32;
  const float4 lw = reinterpret_cast<const float4*>(ln_w)[lane];
  const float4 lb = reinterpret_cast<const float4*>(ln_b)[lane];
  float4 wh[kSHeads];
#pragma unroll
  for (int h = 0; h < kSHeads; ++h) wh[h] = reinterpret_cast<const float4*>(wz + h * 128)[lane];
  float mine[kSHeads];
#pragma unroll
  for (int h = 0; h < kSHeads; ++h) mine[h] = 0.f;
  const int cnt = min(32, rows - i0);
#pragma unroll 1
  for (int ii = 0; ii < cnt; ++ii) {
    const int il = i0 + ii;
    const float4 x =
        __ldg(reinterpret_cast<const float4*>(z_loc + ((size_t)il * n + j) * 128) + lane);
    const float4 y = ln_row_warp(x, lw, lb, eps);
    const float mb = mask ? kSMaskInf * (mask[(size_t)(r0 + il) * n + j] - 1.0f) : 0.f;
#pragma unroll
    for (int h = 0; h < kSHeads; ++h) {
      const float d = warp_sum(y.x * wh[h].x + y.y * wh[h].y + y.z * wh[h].z + y.w * wh[h].w);
      if (lane == ii) mine[h] = d + mb;
    }
  }
  const int il = i0 + lane;
  if (il < rows) {
#pragma unroll
    for (int h = 0; h < kSHeads; ++h) biasT[((size_t)h * n + j) * rows + il] = mine[h];
  }
}

// ---------------------------------------------------------------- attention
// o[i][h*24 + d] for the call's query rows: one thread per query, 64
// queries x one head per block, 32-key tiles of k and v in shared memory
// (every thread reads the same key: broadcasts), online softmax with one
// rescale per tile.
constexpr int kSAttnThreads = 64;

__global__ void __launch_bounds__(kSAttnThreads)
    single_attn_kernel(const float* __restrict__ q, const float* __restrict__ k,
                       const float* __restrict__ v, const float* __restrict__ biasT, int n,
                       int rows, float* __restrict__ o) {
  __shared__ float ks[32][kSDim];
  __shared__ float vs[32][kSDim];
  const int h = blockIdx.y;
  const int il = blockIdx.x * kSAttnThreads + threadIdx.x;
  const bool valid = il < rows;
  const float scale = rsqrtf((float)kSDim);
  float qv[kSDim], ov[kSDim];
#pragma unroll
  for (int d = 0; d < kSDim; ++d) {
    qv[d] = valid ? q[(size_t)il * kCs + h * kSDim + d] * scale : 0.f;
    ov[d] = 0.f;
  }
  float m_run = -INFINITY, l_run = 0.f;
  for (int j0 = 0; j0 < n; j0 += 32) {
    __syncthreads();
    for (int e = threadIdx.x; e < 32 * kSDim; e += kSAttnThreads) {
      const int jj = e / kSDim, d = e % kSDim;
      const int j = j0 + jj;
      ks[jj][d] = j < n ? k[(size_t)j * kCs + h * kSDim + d] : 0.f;
      vs[jj][d] = j < n ? v[(size_t)j * kCs + h * kSDim + d] : 0.f;
    }
    __syncthreads();
    float sc[32];
    float mx = -INFINITY;
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const int j = j0 + jj;
      float s = -INFINITY;
      if (j < n) {
        s = valid ? biasT[((size_t)h * n + j) * rows + il] : 0.f;
#pragma unroll
        for (int d = 0; d < kSDim; ++d) s = fmaf(qv[d], ks[jj][d], s);
      }
      sc[jj] = s;
      mx = fmaxf(mx, s);
    }
    const float m_new = fmaxf(m_run, mx);  // finite: key j0 < n is in the tile
    const float alpha = __expf(m_run - m_new);  // 0 on the first tile
    float ls = 0.f;
#pragma unroll
    for (int d = 0; d < kSDim; ++d) ov[d] *= alpha;
#pragma unroll
    for (int jj = 0; jj < 32; ++jj) {
      const float pj = __expf(sc[jj] - m_new);  // 0 for keys past n
      ls += pj;
#pragma unroll
      for (int d = 0; d < kSDim; ++d) ov[d] = fmaf(pj, vs[jj][d], ov[d]);
    }
    l_run = l_run * alpha + ls;
    m_run = m_new;
  }
  if (valid) {
    const float inv = 1.0f / l_run;
#pragma unroll
    for (int d = 0; d < kSDim; ++d) o[(size_t)il * kCs + h * kSDim + d] = ov[d] * inv;
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
  float *biasT = nullptr, *ta = nullptr, *tb = nullptr;
  void plan(Alloc& al, int n, int rows) {
    a = al.template take<float>((size_t)n * kCs);  // LN(s), all rows
    q = al.template take<float>((size_t)rows * kCs);
    k = al.template take<float>((size_t)n * kCs);
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
  sgemm_nt<kEpiStore>(pl.a, kCs, w->w_k, kCs, pl.k, kCs, n, kCs, kCs, nullptr, stream);
  sgemm_nt<kEpiStore>(pl.a, kCs, w->w_v, kCs, pl.v, kCs, n, kCs, kCs, nullptr, stream);
  sgemm_nt<kEpiSigmoid>(a_mine, kCs, w->w_g, kCs, pl.g, kCs, rows, kCs, kCs, nullptr, stream);
  {
    const long long warps = (long long)n * ((rows + 31) / 32);
    FPB_LAUNCH("single_pair_bias", stream,
               (single_pair_bias_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, stream>>>(
                   z_loc, mask, n, rows, r0, w->ln_z_w, w->ln_z_b, w->w_z, eps, pl.biasT)));
  }
  FPB_LAUNCH("single_attn", stream,
             (single_attn_kernel<<<dim3((rows + kSAttnThreads - 1) / kSAttnThreads, kSHeads),
                                   kSAttnThreads, 0, stream>>>(pl.q, pl.k, pl.v, pl.biasT, n,
                                                               rows, pl.o)));
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
