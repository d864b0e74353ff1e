// Host-side helpers shared by the C-ABI entry points: tensor-map encoding,
// alignment checks and the workspace layout.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stddef.h>
#include <stdint.h>

#include <mutex>

#include "sm100.cuh"

namespace fpb {

// Workspace header: the first 256 bytes of every workspace hold the device
// status word written by bounded waits (0 = ok, else code*1000 + site).
constexpr size_t kWsHeader = 256;

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Bump allocator over a caller-provided workspace (no device allocation).
struct WsCursor {
  uint8_t* base;
  size_t size;
  size_t used;
  bool ok;
  WsCursor(void* b, size_t s) : base(static_cast<uint8_t*>(b)), size(s), used(kWsHeader), ok(true) {}
  template <class T>
  T* take(size_t count) {
    used = align_up(used, 1024);
    T* p = reinterpret_cast<T*>(base + used);
    used += count * sizeof(T);
    if (used > size) ok = false;
    return p;
  }
};

// Counting pass of the same bump allocator (workspace-size queries).
struct WsCounter {
  size_t used = kWsHeader;
  template <class T>
  T* take(size_t count) {
    used = align_up(used, 1024);
    used += count * sizeof(T);
    return nullptr;
  }
};

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D tiled map with 128-byte swizzle: dims {d0 (innermost), d1, d2},
// byte strides {s1, s2} for d1/d2, box {b0, b1, b2}. Out-of-bounds boxes are
// zero-filled. Returns false if the driver rejects the map.
inline bool make_map_3d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                        uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2,
                        uint32_t b0, uint32_t b1, uint32_t b2,
                        CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, b2};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 4-D variant: dims {d0, d1, d2, d3}, byte strides {s1, s2, s3}.
inline bool make_map_4d(CUtensorMap* map, const void* base, CUtensorMapDataType dtype,
                        uint64_t d0, uint64_t d1, uint64_t d2, uint64_t d3, uint64_t s1,
                        uint64_t s2, uint64_t s3, uint32_t b0, uint32_t b1, uint32_t b2,
                        uint32_t b3, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t dims[4] = {d0, d1, d2, d3};
  cuuint64_t strides[3] = {s1, s2, s3};
  cuuint32_t box[4] = {b0, b1, b2, b3};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dtype, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Leading dimension (elements) of a padded row of n entries so that every
// row starts on a 128-byte boundary (TMA strides are 16-byte multiples).
inline int padded_ld(int n, int elem_bytes) {
  const int per = 128 / elem_bytes;
  return (n + per - 1) / per * per;
}

inline int launch_status() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? kOk : kErrCuda;
}

// Opt a kernel in to `bytes` of dynamic shared memory; a refusal is returned
// as kErrCuda (with the CUDA error cleared) instead of surfacing later as a
// less specific launch failure.
template <class Kernel>
inline int set_max_smem(Kernel k, int bytes) {
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess) {
    cudaGetLastError();
    return kErrCuda;
  }
  return kOk;
}

}  // namespace fpb
