// Library-level C-ABI entry points: version, status strings, device checks
// and the workspace status word.
#include "kernels.h"

using namespace fpb;

extern "C" int fpb_abi_version(void) { return 1; }

extern "C" const char* fpb_status_string(int status) {
  switch (status) {
    case kOk: return "ok";
    case kErrShape: return "unsupported shape";
    case kErrAlign: return "misaligned pointer or stride";
    case kErrArg: return "invalid argument";
    case kErrCuda: return "CUDA launch error";
    case kErrTimeout: return "device-side wait timed out";
    case kErrWorkspace: return "workspace too small";
    case kErrScratch: return "request exceeds the static scratch capacity";
    default: return "unknown status";
  }
}

// 0 when `device` is an sm_100 (B200-class) GPU, kErrArg otherwise.
extern "C" int fpb_device_supported(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess)
    return kErrCuda;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess)
    return kErrCuda;
  return (major == 10 && minor == 0) ? kOk : kErrArg;
}

// Synchronises `stream` and reads the device status word of a workspace:
// 0 when every bounded wait of the calls that used it completed, otherwise
// code * 1000 + site of the first failure.
extern "C" int fpb_workspace_status(const void* workspace, cudaStream_t stream, int* out_status) {
  if (!workspace || !out_status) return kErrArg;
  int v = 0;
  if (cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return kErrCuda;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return kErrCuda;
  *out_status = v;
  return kOk;
}
