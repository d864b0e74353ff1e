// Peer-memory exchange helpers for the row-sharded block on the GPUs of one
// node (one process per GPU). A rank exports a device buffer as a CUDA IPC
// handle plus its offset inside the allocation; the other ranks map it into
// their own context (peer access enabled lazily) and copy their blocks
// straight into it over NVLink, so an all-to-all or all-gather needs no
// staging copy and no collective protocol beyond an ordering barrier.
// Nothing here allocates device memory: the buffers belong to the caller.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstring>
#include <mutex>

#include "kernels.h"
#include "../../include/fireprot_b200.h"

namespace fpb {
namespace {

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

constexpr int kMaxPeers = 16;
struct PeerDst {
  float4* p[kMaxPeers];
};

// One warp per (i, j) pair of the rank's rows: the ch floats of z[i, j] are
// contiguous in z_loc and land contiguous in row (j - d*chunk), column
// r0 + i of rank d's [chunk][n][ch] buffer, so both sides move whole
// 512-byte vectors (ch = 128) and a warp's store is one NVLink burst.
// Four pairs per iteration keep four independent HBM loads in flight.
__global__ void __launch_bounds__(256) peer_transpose_kernel(const float4* __restrict__ z, int n,
                                                             int chunk, int r0, int rows,
                                                             int ch4, PeerDst dst) {
  const int lane = threadIdx.x & 31;
  const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const long long pairs = static_cast<long long>(rows) * n;
  for (long long p0 = warp; p0 < pairs; p0 += 4 * nwarps) {
    for (int c4 = lane; c4 < ch4; c4 += 32) {
      float4 v[4];
      float4* out[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const long long p = p0 + u * nwarps;
        out[u] = nullptr;
        if (p < pairs) {
          const int i = static_cast<int>(p / n);
          const int j = static_cast<int>(p - static_cast<long long>(i) * n);
          const int d = j / chunk;
          out[u] = dst.p[d] + (static_cast<size_t>(j - d * chunk) * n + r0 + i) * ch4 + c4;
          v[u] = __ldcs(z + static_cast<size_t>(p) * ch4 + c4);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (out[u]) *out[u] = v[u];
    }
  }
}

struct CopySeg {
  const float4* src;
  float4* dst;
  long long n4;
};
struct CopySegs {
  CopySeg s[kMaxPeers];
};

// Block row y copies segment y; its blocks stride over the segment with
// four independent 16-byte loads in flight per thread before the stores, so
// every peer's NVLink port is written by SMs at once (the copy engines run
// one transfer per engine, and a few engines cannot fill the fabric).
__global__ void __launch_bounds__(256) peer_scatter_kernel(CopySegs segs) {
  const CopySeg sg = segs.s[blockIdx.y];
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < sg.n4; i += 4 * stride) {
    const float4 v0 = __ldcs(sg.src + i);
    const float4 v1 = __ldcs(sg.src + i + stride);
    const float4 v2 = __ldcs(sg.src + i + 2 * stride);
    const float4 v3 = __ldcs(sg.src + i + 3 * stride);
    sg.dst[i] = v0;
    sg.dst[i + stride] = v1;
    sg.dst[i + 2 * stride] = v2;
    sg.dst[i + 3 * stride] = v3;
  }
  for (; i < sg.n4; i += stride) sg.dst[i] = __ldcs(sg.src + i);
}

}  // namespace
}  // namespace fpb

using namespace fpb;

extern "C" int fpb_peer_scatter(const void* const* src, void* const* dst, const size_t* bytes,
                                int count, cudaStream_t stream) {
  if (count < 0 || count > kMaxPeers || (count && (!src || !dst || !bytes))) return kErrArg;
  CopySegs segs{};
  int used = 0;
  for (int k = 0; k < count; ++k) {
    if (!bytes[k]) continue;
    if (!src[k] || !dst[k] || !aligned16(src[k]) || !aligned16(dst[k]) || (bytes[k] & 15))
      return kErrArg;
    segs.s[used++] = CopySeg{static_cast<const float4*>(src[k]), static_cast<float4*>(dst[k]),
                             static_cast<long long>(bytes[k] / 16)};
  }
  if (!used) return kOk;
  const int per = (sm_count() * 8 + used - 1) / used;  // 8 blocks of 256 per SM in all
  FPB_LAUNCH("peer_scatter", stream,
             peer_scatter_kernel<<<dim3(static_cast<unsigned>(per), static_cast<unsigned>(used)),
                                   256, 0, stream>>>(segs));
  return launch_status();
}

extern "C" int fpb_peer_transpose_rows(const float* z_loc, int n, int chunk, int ch, int rank,
                                       int world, float* const* dst, cudaStream_t stream) {
  if (!z_loc || !dst || n <= 0 || chunk <= 0 || ch <= 0 || (ch & 3) || world <= 0 ||
      world > kMaxPeers || rank < 0 || rank >= world ||
      static_cast<long long>(chunk) * world < n || !aligned16(z_loc))
    return kErrArg;
  PeerDst pd{};
  for (int d = 0; d < world; ++d) {
    // every rank that owns a column of z also receives rows
    if (d * chunk < n && (!dst[d] || !aligned16(dst[d]))) return kErrArg;
    pd.p[d] = reinterpret_cast<float4*>(dst[d]);
  }
  const int r0 = rank * chunk;
  const int rows = r0 >= n ? 0 : (n - r0 < chunk ? n - r0 : chunk);
  if (rows == 0) return kOk;
  const long long pairs = static_cast<long long>(rows) * n;
  long long grid = (pairs + 31) / 32;  // 8 warps a block, 4 pairs a warp
  const long long cap = static_cast<long long>(sm_count()) * 8;
  if (grid > cap) grid = cap;
  FPB_LAUNCH("peer_transpose", stream,
             peer_transpose_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(
                 reinterpret_cast<const float4*>(z_loc), n, chunk, r0, rows, ch / 4, pd));
  return launch_status();
}

extern "C" size_t fpb_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int fpb_ipc_export(const void* ptr, void* handle_out, size_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return kErrArg;
  auto range = address_range_fn();
  if (!range) return kErrCuda;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return kErrArg;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) {
    cudaGetLastError();
    return kErrCuda;
  }
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base);
  return kOk;
}

extern "C" int fpb_ipc_import(const void* handle, size_t offset, void** base_out,
                              void** ptr_out) {
  if (!handle || !base_out || !ptr_out) return kErrArg;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return kErrCuda;
  }
  *base_out = base;
  *ptr_out = static_cast<uint8_t*>(base) + offset;
  return kOk;
}

extern "C" int fpb_ipc_close(void* base) {
  if (!base) return kErrArg;
  if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
    cudaGetLastError();
    return kErrCuda;
  }
  return kOk;
}

extern "C" int fpb_copy_async(void* dst, const void* src, size_t bytes, cudaStream_t stream) {
  if ((!dst || !src) && bytes) return kErrArg;
  if (!bytes) return kOk;
  if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, stream) != cudaSuccess) {
    cudaGetLastError();
    return kErrCuda;
  }
  return kOk;
}
