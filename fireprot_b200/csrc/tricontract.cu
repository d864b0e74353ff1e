// Triangle contraction on channels-last tensors, the ESMFold2 form
// (TriangleMultiplicativeBlock._triangular_contract_chunked, as the
// reference's python/fireprot/adapters/esmfold2/triangle.py:19-33 dispatches
// it; ESMFold2 uses C = 256 channels):
//   outgoing: x[i][j][c] = sum_k left[i][k][c] right[j][k][c]
//   incoming: x[i][j][c] = sum_k left[k][i][c] right[k][j][c]
// left, right, x: [n][n][C] FP32. The operands are transposed through
// shared memory into the channel-first, K-major hi/lo (strict) or BF16
// (fast) planes of the batched contraction kernel, which writes x in its
// blocked layout [i][j / 128][c][j % 128]; a second transpose turns each
// [C][128] block back into 128 channels-last rows.
#include "../../include/fireprot_b200.h"
#include "kernels.h"

namespace fpb {

// One block: 32 keys k x 32 channels c of one row i. Reads are 128-byte
// channel runs src[i * si + k * sk + c0 .. c0 + 31]; writes are 128-byte runs
// of plane c along k.
template <bool kStrict>
__global__ void pack_cl_kernel(const float* __restrict__ src, int n, long long si, long long sk,
                               void* __restrict__ hi, void* __restrict__ lo, int ld,
                               size_t cstride) {
  __shared__ float tile[32][33];
  const int k0 = blockIdx.x * 32, c0 = blockIdx.y * 32, i = blockIdx.z;
  const int tx = threadIdx.x;
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    const int k = k0 + y;
    tile[y][tx] = k < n ? src[(long long)i * si + (long long)k * sk + c0 + tx] : 0.f;
  }
  __syncthreads();
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    const int c = c0 + y, k = k0 + tx;
    if (k >= n) continue;
    const float v = tile[tx][y];
    const size_t idx = (size_t)c * cstride + (size_t)i * ld + k;
    if constexpr (kStrict) {
      float h, l;
      split_tf32(v, h, l);
      static_cast<float*>(hi)[idx] = h;
      static_cast<float*>(lo)[idx] = l;
    } else {
      static_cast<__nv_bfloat16*>(hi)[idx] = __float2bfloat16_rn(v);
    }
  }
}

// blocked [i][jb][c][128] -> channels-last out[i][jb * 128 + jj][c]. One
// block: 32 columns jj x 32 channels of one (i, jb).
__global__ void unblock_cl_kernel(const float* __restrict__ blk, int n, int channels, int njb,
                                  float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int jb = blockIdx.x / 4, jq = (blockIdx.x % 4) * 32;
  const int c0 = blockIdx.y * 32, i = blockIdx.z;
  const int tx = threadIdx.x;
  const float* base = blk + (((size_t)i * njb + jb) * channels) * 128;
  for (int y = threadIdx.y; y < 32; y += blockDim.y)
    tile[y][tx] = base[(size_t)(c0 + y) * 128 + jq + tx];  // [c][jj]
  __syncthreads();
  for (int y = threadIdx.y; y < 32; y += blockDim.y) {
    const int j = jb * 128 + jq + y;
    if (j < n) out[((size_t)i * n + j) * channels + c0 + tx] = tile[tx][y];
  }
}

template <class Alloc>
struct TriContractPlan {
  void *a_hi = nullptr, *a_lo = nullptr, *b_hi = nullptr, *b_lo = nullptr;
  float* x = nullptr;
  int ld = 0, njb = 0;
  size_t cs = 0;
  void plan(Alloc& al, int n, int channels, bool strict) {
    const int esz = strict ? 4 : 2;
    ld = padded_ld(n, esz);
    cs = (size_t)n * ld;
    njb = (n + 127) / 128;
    auto take = [&](size_t c) -> void* {
      return strict ? (void*)al.template take<float>(c) : (void*)al.template take<__nv_bfloat16>(c);
    };
    const size_t count = (size_t)channels * cs;
    a_hi = take(count);
    if (strict) a_lo = take(count);
    b_hi = take(count);
    if (strict) b_lo = take(count);
    x = al.template take<float>((size_t)n * njb * channels * 128);
  }
};

}  // namespace fpb

using namespace fpb;

extern "C" size_t fpb_triangle_contract_workspace_size(int n, int channels, int precision) {
  if (n <= 0 || channels <= 0 || channels % 32 || (precision != 0 && precision != 1)) return 0;
  WsCounter cnt;
  TriContractPlan<WsCounter> pl;
  pl.plan(cnt, n, channels, precision == 0);
  return cnt.used;
}

extern "C" int fpb_triangle_contract(const float* left, const float* right, float* out, int n,
                                     int channels, int outgoing, int precision, void* workspace,
                                     size_t workspace_bytes, cudaStream_t stream) {
  if (!left || !right || !out || !workspace) return kErrArg;
  if (precision != 0 && precision != 1) return kErrArg;
  if (n <= 0 || channels <= 0 || channels % 32 || channels > 65535) return kErrShape;
  if (!aligned16(left) || !aligned16(right) || !aligned16(out) || !aligned16(workspace))
    return kErrAlign;
  if (workspace_bytes < fpb_triangle_contract_workspace_size(n, channels, precision))
    return kErrWorkspace;
  const bool strict = precision == 0;
  WsCursor cur(workspace, workspace_bytes);
  TriContractPlan<WsCursor> pl;
  pl.plan(cur, n, channels, strict);
  if (!cur.ok) return kErrWorkspace;
  if (reset_status(workspace, stream)) return kErrCuda;
  // A_c[i][k] = left at (i, k) (outgoing) or (k, i) (incoming); B likewise
  const long long row = (long long)n * channels;
  const long long si = outgoing ? row : channels, sk = outgoing ? channels : row;
  const dim3 pg((n + 31) / 32, channels / 32, n), pb(32, 8);
  if (strict) {
    FPB_LAUNCH("tricontract_pack", stream,
               (pack_cl_kernel<true><<<pg, pb, 0, stream>>>(left, n, si, sk, pl.a_hi, pl.a_lo,
                                                            pl.ld, pl.cs)));
    FPB_LAUNCH("tricontract_pack", stream,
               (pack_cl_kernel<true><<<pg, pb, 0, stream>>>(right, n, si, sk, pl.b_hi, pl.b_lo,
                                                            pl.ld, pl.cs)));
  } else {
    FPB_LAUNCH("tricontract_pack", stream,
               (pack_cl_kernel<false><<<pg, pb, 0, stream>>>(left, n, si, sk, pl.a_hi, nullptr,
                                                             pl.ld, pl.cs)));
    FPB_LAUNCH("tricontract_pack", stream,
               (pack_cl_kernel<false><<<pg, pb, 0, stream>>>(right, n, si, sk, pl.b_hi, nullptr,
                                                             pl.ld, pl.cs)));
  }
  int st;
  if ((st = launch_status())) return st;
  ContractOperands op{pl.a_hi, pl.a_lo, pl.b_hi, pl.b_lo, pl.ld, pl.cs, pl.cs, n, n, n,
                      n,       1,        0,        channels, strict};
  ContractArgs args{};
  args.out = pl.x;
  args.out_bf16 = 0;
  args.status = static_cast<int*>(workspace);
  args.blocked = 1;
  args.njb = pl.njb;
  args.bchannels = channels;
  if ((st = launch_contract(op, args, stream))) return st;
  FPB_LAUNCH("tricontract_unpack", stream,
             (unblock_cl_kernel<<<dim3(pl.njb * 4, channels / 32, n), dim3(32, 8), 0, stream>>>(
                 pl.x, n, channels, pl.njb, out)));
  return launch_status();
}
