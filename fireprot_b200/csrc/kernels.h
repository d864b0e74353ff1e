// Internal launch interfaces shared between the translation units of the
// library (not part of the public C ABI).
#pragma once

#include "host_common.h"

namespace fpb {

// Operands of the batched contraction X_c = A_c B_c^T (K-major, padded rows).
struct ContractOperands {
  const void* a_hi;
  const void* a_lo;  // strict only
  const void* b_hi;
  const void* b_lo;  // strict only
  int ld;                 // row pitch of A/B (elements)
  size_t channel_stride;  // elements between channels
  int channels;
  bool strict;
};

struct ContractArgs {
  int n;
  void* out;                  // [channels][n][ldo] fp32 or bf16
  int ldo;
  size_t out_channel_stride;  // elements
  int out_bf16;
  int* status;
};

int launch_contract(const ContractOperands& op, const ContractArgs& args, cudaStream_t stream);

}  // namespace fpb
