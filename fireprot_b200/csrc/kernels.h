// Internal launch interfaces shared between the translation units of the
// library (not part of the public C ABI).
#pragma once

#include "host_common.h"

namespace fpb {

// Operands of the batched contraction X_c = A_c B_c^T (K-major, padded rows):
// A_c is [m][k], B_c is [nn][k]. B may be a rank-major all-gather buffer:
// b_chunks chunks of b_chunk_rows rows each, b_chunk_stride elements apart,
// each chunk laid out [channel][row][ld]; rows of the last chunk at or past
// nn (padding of a ragged split) are read but never stored.
struct ContractOperands {
  const void* a_hi;
  const void* a_lo;  // strict only
  const void* b_hi;
  const void* b_lo;  // strict only
  int ld;                   // row pitch of A and B (elements)
  size_t a_channel_stride;  // elements between A channels
  size_t b_channel_stride;  // elements between B channels (within a chunk)
  int m, nn, k;
  int b_chunk_rows;
  int b_chunks;
  size_t b_chunk_stride;
  int channels;
  bool strict;
};

struct ContractArgs {
  int m, nn, k;  // filled by launch_contract from the operands
  int bn;        // column tile (32..256)
  int b_chunk_rows;
  void* out;                  // [channels][n][ldo] fp32 or bf16 (plain layout)
  int ldo;
  size_t out_channel_stride;  // elements
  int out_bf16;
  int* status;
  // blocked layout (when blocked != 0): out[i][j / 128][c][j % 128] with
  // njb = ceil(n / 128) column blocks; one pair-row tile of the output
  // kernel (128 columns x all channels) is then one contiguous block.
  int blocked;
  int njb;
  int bchannels;  // channels per block of the blocked layout (0: 128)
  // Owner scatter (blocked layout, owners > 0): output row r is stored in
  // outs[r / owner_rows] at row r % owner_rows of a blocked layout of 128
  // channels, channel ch + ch_off: every row goes straight to the x buffer
  // of the rank that owns it (a peer address for the other ranks).
  int owners;
  int owner_rows;
  int ch_off;
  void* outs[16];
};

int launch_contract(const ContractOperands& op, const ContractArgs& args, cudaStream_t stream);

// Zero the workspace status word at the start of a public call, unless the
// call runs inside a composite call (fpb_pair_block) that owns the word.
int reset_status(void* workspace, cudaStream_t stream);
struct CompositeCall {
  CompositeCall();
  ~CompositeCall();
};

// Launch timing (timing.cu): bracket a kernel launch with CUDA events when
// timing is enabled on this thread.
int timing_begin(cudaStream_t s);
void timing_end(int idx, cudaStream_t s, const char* name);

#define FPB_LAUNCH(name, stream, ...)                  \
  do {                                                 \
    const int fpb_t_ = ::fpb::timing_begin(stream);    \
    __VA_ARGS__;                                       \
    ::fpb::timing_end(fpb_t_, stream, name);           \
  } while (0)

// Concatenate up to 4 [rows_each][128] FP32 weight matrices and split them
// into tf32 hi/lo (strict) or convert them to BF16 (fast).
struct PackSrc {
  const float* m[4];
  int count;
  int rows_each;
};
int pack_weights(const PackSrc& src, void* hi, void* lo, bool strict, cudaStream_t stream);

// TMA maps over packed weights [rows][128], one 128-byte K atom x 128 rows per box.
bool make_weight_maps(const void* hi, const void* lo, int rows, bool strict, CUtensorMap* mh,
                      CUtensorMap* ml);

// Number of SMs of the current device (cached per device): the grid of a
// persistent kernel (one CTA per SM walking tiles).
int sm_count();

// Dynamic shared memory to request so that the number of co-resident CTAs
// never exceeds what TMEM can hold (512 columns per SM): a CTA never waits
// inside tcgen05.alloc.
constexpr int tmem_safe_smem(int need, int tmem_cols) {
  const int max_ctas = 512 / tmem_cols;
  const int floor_bytes = (228 * 1024) / (max_ctas + 1) + 1024;
  return need > floor_bytes ? need : floor_bytes;
}

}  // namespace fpb
