/*
 * fireprot_b200 — C ABI of the B200 (sm_100a) backend for the Pairformer
 * pair-representation hot path.
 *
 * Conventions (mirroring the reference's C-ABI kernels):
 *  - every entry point returns an int status: 0 ok, 2 unsupported shape,
 *    3 misaligned pointer/stride, 4 invalid argument, 5 CUDA launch error,
 *    6 device-side wait timed out, 7 workspace too small, 8 request exceeds
 *    the static scratch capacity (fpb_transition_noalloc only)
 *    (reference: kernels/amd/fireprot_ck_attention.cpp:35,68,106-108,
 *    kernels/amd/fireprot_lt_bmm.cpp:47-48,62);
 *  - pointers are raw device pointers, work is enqueued on `stream`, nothing
 *    is allocated: the caller passes a workspace of at least the size the
 *    matching *_workspace_size function returns (16-byte aligned); its first
 *    256 bytes hold a device status word (see fpb_workspace_status);
 *  - `precision`: 0 = strict FP32 (3xTF32 tensor-core products),
 *    1 = fast (BF16 operands, FP32 accumulation);
 *  - pair tensors are [N, N, C] FP32, C-contiguous (channels last), masks
 *    [N, N] FP32 with 1 = valid (nullable: no mask).
 */
#ifndef FIREPROT_B200_H
#define FIREPROT_B200_H

#include <stddef.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FPB_STRICT 0
#define FPB_FAST 1

/* ABI version of this library (1). Reference: the Rust bridge's ABI gate,
 * python/fireprot/ops/_bridge.py:32-33. */
int fpb_abi_version(void);

/* Human-readable text for a status code. */
const char* fpb_status_string(int status);

/* 0 when `device` is an sm_100 GPU. */
int fpb_device_supported(int device);

/* Synchronise `stream`, then read the device status word of `workspace`. */
int fpb_workspace_status(const void* workspace, cudaStream_t stream, int* out_status);

/* Batched triangle contraction over `batch` channel planes of n x n FP32:
 * outgoing: out[c] = a[c] @ b[c]^T; incoming: out[c] = a[c]^T @ b[c].
 * Replaces lt_packed_bmm (kernels/amd/fireprot_lt_bmm.cpp:46-63, Python
 * caller python/fireprot/backends/amd/lt_bmm.py:65-85) for any n and batch;
 * a, b, out contiguous [batch, n, n]. */
size_t fpb_packed_bmm_workspace_size(int batch, int n, int precision);
int fpb_packed_bmm(const float* a, const float* b, float* out, int batch, int n, int outgoing,
                   int precision, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Triangle multiplicative update, whole operator, in place on z [n, n, 128]:
 *   zn = LN_in(z); a = mask*sigmoid(zn Wag^T)*(zn Wap^T); b likewise;
 *   outgoing x_ij = sum_k a_ik b_jk, incoming x_ij = sum_k a_ki b_kj;
 *   z <- [z +] sigmoid(zn Wg^T) * (LN_out(x) Wz^T)   (add = 1 / 0).
 * Weights are torch Linear layouts [out, in] FP32 (bias-free), LN params
 * [128]. Replaces the packed path of dispatch_triangle_multiplication
 * (python/fireprot/backends/amd/triangle_multiplication.py:296-344, selected
 * at :389-430) and its kernels dual_projection_tiled / lt_packed_bmm /
 * packed_norm_vector / triangle_residual (kernels/amd/fireprot_amd_ops.cu:
 * 594-646,663-708,787-863; kernels/amd/fireprot_lt_bmm.cpp:46-63).
 * z and the LN_in parameters must be 16-byte aligned. */
size_t fpb_trimul_workspace_size(int n, int c_z, int precision);
int fpb_trimul(float* z, const float* mask, int n, int c_z, const float* ln_in_w,
               const float* ln_in_b, const float* w_a_p, const float* w_a_g, const float* w_b_p,
               const float* w_b_g, const float* w_g, const float* ln_out_w, const float* ln_out_b,
               const float* w_z, float eps, int outgoing, int add, int precision, void* workspace,
               size_t workspace_bytes, cudaStream_t stream);

/* Triangle attention (starting node when starting = 1, ending node when 0),
 * whole operator, residual added in place: z <- z + delta with
 *   x = LN(y), y = z (start) or z^T (end, mask^T);
 *   s_ijk = (x_ij Wq_h^T/sqrt(d)) . (x_ik Wk_h^T) + 1e9 (mask_ik - 1) + x_jk . Wbias_h
 *   o_ij = sum_k softmax_k(s) (x_ik Wv_h^T); delta = W_o (sigmoid(x Wg^T + b_g) * o) + b_o
 * (end node: delta transposed back). With delta_out non-null the update is
 * written there ([n, n, 128], the reference module's return value) and z is
 * left unchanged. heads = 4, head_dim = 32, c_z = 128;
 * w_q/w_k/w_v/w_g [128,128], w_bias [4,128], w_o [128,128]; b_g, b_o nullable.
 * Replaces dispatch_triangle_attention + the QKV / gate hooks
 * (python/fireprot/backends/amd/triangle_attention.py:199-256,
 * qkv_projection.py:54-66, attention_gate.py:28-56) and their kernels
 * project_qkv / ck_attention* / sigmoid_mul_out (kernels/amd/fireprot_amd_ops.cu:
 * 537-565,871-955; kernels/amd/fireprot_ck_attention.cpp:34-121).
 * The mask bias follows patches/protenix/0005-...patch:35-38 (inf = 1e9). */
size_t fpb_triattn_workspace_size(int n, int c_z, int heads, int head_dim, int precision,
                                  int with_mask);
int fpb_triattn(float* z, float* delta_out, const float* mask, int n, int c_z, int heads,
                int head_dim,
                const float* ln_w, const float* ln_b, const float* w_q, const float* w_k,
                const float* w_v, const float* w_bias, const float* w_g, const float* b_g,
                const float* w_o, const float* b_o, float eps, int starting, int precision,
                void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Pair transition, residual added in place on `rows` rows of 128 channels:
 *   z <- z + (silu(LN(z) Wa^T) * (LN(z) Wb^T)) Wout^T
 * expansion = 4: w_a, w_b [512,128], w_out [128,512], bias-free. With delta_out
 * non-null the update alone is written there (the reference's
 * Transition.forward return value) and z is left unchanged.
 * Replaces dispatch_transition / _hip_transition
 * (python/fireprot/backends/amd/recycle.py:203-227,360) and the
 * project_transition kernel (kernels/amd/fireprot_amd_ops.cu:1106-1183). */
size_t fpb_transition_workspace_size(int c_z, int expansion, int precision);
int fpb_transition(float* z, float* delta_out, long long rows, int c_z, int expansion,
                   const float* ln_w, const float* ln_b, const float* w_a, const float* w_b,
                   const float* w_out, float eps, int precision, void* workspace,
                   size_t workspace_bytes, cudaStream_t stream);

/* Allocation-free pair transition. No counterpart in the reference: it is
 * fpb_transition (same kernels, same results) for callers that must not
 * allocate device memory, such as a serving process whose memory manager
 * reserves the GPU's memory up front and owns every later allocation (a
 * cudaMalloc from a library would then fail or break its accounting, and
 * cudaFree synchronises the whole device), or a host behind an FFI with no
 * device allocator of its own, which would need one only for this scratch.
 *
 * The scratch (packed weights plus the 256-byte status word) is a static
 * device array of this library, FPB_TRANSITION_SCRATCH_BYTES per device; a
 * request needing more is rejected with status 8. Nothing else is allocated.
 *  - Every call looks up the array's device address in the current device's
 *    current context (the address is per context, so it is never cached).
 *    The first call on a device may load the library's device code there:
 *    make that first call before any stream capture that would include
 *    this function.
 *  - Each call zeroes the status word on `stream` before its kernels (the
 *    only part that must start at zero) and overwrites the packed weights.
 *  - Calls on one device share the array: calls that can overlap (several
 *    streams or threads on one device) race and must be serialised by the
 *    caller, e.g. by issuing them on one stream.
 *  - status_out (nullable host pointer): when given, the call waits for
 *    `stream` and stores the device status word (0 = every wait completed,
 *    else 6000 + site of a device-side wait that timed out). Waiting is
 *    illegal while `stream` is being captured, so a non-null status_out on a
 *    capturing stream is rejected with status 4. With status_out null the
 *    call never reports a device-side timeout: the word stays in the static
 *    array, which the caller cannot read through this API.
 * Arguments otherwise as fpb_transition; z, the weights and `stream` belong
 * to the current device. */
#define FPB_TRANSITION_SCRATCH_BYTES (2u << 20)
int fpb_transition_noalloc(float* z, float* delta_out, long long rows, int c_z, int expansion,
                           const float* ln_w, const float* ln_b, const float* w_a,
                           const float* w_b, const float* w_out, float eps, int precision,
                           int* status_out, cudaStream_t stream);

/* Triangle attention core at the reference's q/k/v boundary
 * (dispatch_triangle_attention, python/fireprot/backends/amd/triangle_attention.py:199-256,
 * replacing ck_attention* in kernels/amd/fireprot_ck_attention.cpp:34-121):
 *   out[b, j, h, :] = sum_k softmax_k(q[b,h,j,:].k[b,h,k,:] + mask_bias[b,0,0,k]
 *                                     + tri_bias[0,h,j,k]) v[b,h,k,:]
 * q (already scaled), k, v: [batch, 4, n, 32] FP32 with element strides
 * (4 entries each); tri_bias [1, 4, n, n], mask_bias [batch, 1, 1, n] or null,
 * any strides; out [batch, n, 4, 32] contiguous FP32 (both precisions).
 * -inf biases are exact: such keys get weight 0. A query row whose every
 * logit is -inf gives 0, as the torch scaled_dot_product_attention the
 * reference's dispatch checks against (triangle_attention.py:83-129, tested
 * with a -inf bias row at tests/operators/test_ck_attention.py:69-81). */
size_t fpb_attention_core_workspace_size(int batch, int n, int heads, int head_dim,
                                         int precision, int with_mask);
int fpb_attention_core(const float* q, const long long* q_strides, const float* k,
                       const long long* k_strides, const float* v, const long long* v_strides,
                       int batch, int n, int heads, int head_dim, const float* tri_bias,
                       const long long* tri_bias_strides, const float* mask_bias,
                       const long long* mask_bias_strides, float* out, int precision,
                       void* workspace, size_t workspace_bytes, cudaStream_t stream);
/* fpb_attention_core with the result of an all -inf row chosen:
 * empty_rows_nan = 0 gives 0 (as fpb_attention_core), 1 gives NaN, the
 * contract of the OpenFold3 mask + bias softmax that a zero row sum is NaN
 * (kernels/amd/fireprot_softmax_fp32.cpp:61-62, followed by upstream's P V
 * einsum; python/fireprot/adapters/openfold3/attention.py:135-148). */
int fpb_attention_core_ex(const float* q, const long long* q_strides, const float* k,
                          const long long* k_strides, const float* v,
                          const long long* v_strides, int batch, int n, int heads, int head_dim,
                          const float* tri_bias, const long long* tri_bias_strides,
                          const float* mask_bias, const long long* mask_bias_strides, float* out,
                          int precision, int empty_rows_nan, void* workspace,
                          size_t workspace_bytes, cudaStream_t stream);

/* Operator policy registry (host only), the counterpart of the reference's
 * Rust core crates/fireprot-core/src/registry.rs:95-268 behind its bridge
 * protocol (crates/fireprot-bridge/src/lib.rs:86-125): JSON metadata and
 * signatures in, JSON selections and manifests out. Capability callbacks
 * return 1 (supported), 0 (rejected, reason written) or -1 (interrupted). */
typedef int (*fpb_capability_fn)(const char* signature_json, void* user, char* reason,
                                 size_t cap);
void* fpb_registry_new(void);
void fpb_registry_free(void* registry);
int fpb_registry_register(void* registry, const char* metadata_json, fpb_capability_fn fn,
                          void* user);
int fpb_registry_unregister(void* registry, const char* operation, const char* name);
int fpb_registry_resolve(void* registry, const char* signature_json, char* out, size_t cap);
int fpb_registry_manifest(void* registry, char* out, size_t cap);
int fpb_registry_clear_runtime_state(void* registry);

/* ---- Row-sharded phases (one rank owns rows [r0, r0 + rows) of z; the
 * caller runs the NCCL collectives between phases). These split the fused
 * operators above at their exchange points; the reference has no multi-GPU
 * path for these operators (its only multi-device code is the two-GCD
 * outer-batch split, python/fireprot/backends/amd/two_gcd_attention.py:53-101).
 *
 * TriMul planes are channel-first [128][plane_rows][ld] (ld =
 * fpb_trimul_plane_ld of the column count), FP32 hi and lo in strict mode,
 * BF16 in fast mode; the contraction output is tile-blocked
 * [m][ceil(nn/128)][128][128] (FP32 strict, BF16 fast).
 *   outgoing: proj(transposed=0, plane_rows=chunk) -> all-gather b ->
 *             contract(m=rows, nn=n, B = the gathered chunks, k=n) -> finish.
 *   incoming: proj(transposed=1, plane_rows=n) -> contract(m=n, nn=n, one B
 *             chunk of n rows, k=rows) -> reduce-scatter x -> finish.
 * In an all-gather buffer the chunk height must be a multiple of 32 rows;
 * rows of the last chunk at or past nn are padding and are never stored. */
size_t fpb_trimul_shard_workspace_size(int precision);
size_t fpb_trimul_plane_ld(int cols, int precision);
int fpb_trimul_shard_proj(const float* z_loc, const float* mask, int n, int rows, int r0,
                          int transposed, const float* ln_in_w, const float* ln_in_b,
                          const float* w_a_p, const float* w_a_g, const float* w_b_p,
                          const float* w_b_g, float eps, void* a_hi, void* a_lo, void* b_hi,
                          void* b_lo, int ld, int plane_rows, int precision, void* workspace,
                          size_t workspace_bytes, cudaStream_t stream);
/* Strict mode may pass a_lo and/or b_lo = NULL to fpb_trimul_shard_proj: a
 * or b is then written unsplit (FP32) into its hi planes, half the bytes of
 * the exchange that follows; after it, fpb_split_tf32 splits the received
 * planes exactly (hi = x with the low 13 mantissa bits cleared, lo = x - hi;
 * hi may alias src). No reference counterpart (the reference has no sharded
 * path). */
int fpb_split_tf32(const float* src, void* hi, void* lo, size_t count, cudaStream_t stream);
int fpb_trimul_shard_contract(const void* a_hi, const void* a_lo, int m, int a_plane_rows,
                              const void* b_hi, const void* b_lo, int nn, int b_chunk_rows,
                              int b_chunks, size_t b_chunk_stride, int k, int ld,
                              void* x_blocked, int precision, void* workspace,
                              size_t workspace_bytes, cudaStream_t stream);
/* Channel-group form of the contraction (the channel-sharded TriMul: every
 * rank projects its rows, an all-to-all hands channel group g of every rank's
 * planes to rank g, which contracts its `channels` planes over the whole
 * n x n grid; a second all-to-all returns the output rows). The operands are
 * `channels` planes laid out as for fpb_trimul_shard_contract; the output is
 * blocked [m][ceil(nn/128)][channels][128]. fpb_trimul_shard_contract is this
 * call with channels = 128. */
int fpb_trimul_group_contract(const void* a_hi, const void* a_lo, int m, int a_plane_rows,
                              const void* b_hi, const void* b_lo, int nn, int b_chunk_rows,
                              int b_chunks, size_t b_chunk_stride, int k, int ld, int channels,
                              void* x_blocked, int precision, void* workspace,
                              size_t workspace_bytes, cudaStream_t stream);
/* fpb_trimul_shard_proj for the channel-group exchange with a and b stored
 * straight at their owners: channel c of a (b) goes to a_owner[c / G]
 * (b_owner[c / G]), G = 128 / owners, plane rank * G + c % G of that
 * rank's [owners][G][plane_rows][ld] receive buffer (a peer mapping for the
 * other ranks), unsplit in strict mode. Columns or rows the call does not
 * own are not written. The caller orders the stores against the owners'
 * reads (a barrier after the call; the buffers' previous readers must have
 * passed a barrier before it). */
int fpb_trimul_shard_proj_scatter(const float* z_loc, const float* mask, int n, int rows, int r0,
                                  int transposed, const float* ln_in_w, const float* ln_in_b,
                                  const float* w_a_p, const float* w_a_g, const float* w_b_p,
                                  const float* w_b_g, float eps, void* const* a_owner,
                                  void* const* b_owner, int owners, int rank, int ld,
                                  int plane_rows, int precision, void* workspace,
                                  size_t workspace_bytes, cudaStream_t stream);
/* fpb_trimul_group_contract with the output rows stored straight at their
 * owners: output row r goes to x_owner[r / owner_rows] (owners <= 16
 * pointers, a peer mapping for the other ranks' buffers) at row
 * r % owner_rows of the blocked [owner_rows][ceil(nn/128)][128][128]
 * layout, channel c + ch_off. Rank g of the channel-sharded TriMul passes
 * ch_off = g * channels, so every rank's buffer ends up holding all 128
 * channels of its rows, the layout fpb_trimul_shard_finish reads, with no
 * return exchange and no regrouping pass. The caller orders the stores
 * against the owners' reads (a barrier before and after). */
int fpb_trimul_group_contract_scatter(const void* a_hi, const void* a_lo, int m, int a_plane_rows,
                                      const void* b_hi, const void* b_lo, int nn,
                                      int b_chunk_rows, int b_chunks, size_t b_chunk_stride,
                                      int k, int ld, int channels, void* const* x_owner,
                                      int owners, int owner_rows, int ch_off, int precision,
                                      void* workspace, size_t workspace_bytes,
                                      cudaStream_t stream);
/* Operand gather of the channel-group exchange: src is the all-to-all
 * receive buffer [world][channels][rows][src_ld] (FP32 unsplit in strict
 * mode, BF16 in fast mode); the call writes the contraction operand, split
 * into hi/lo (strict) or copied (fast) in the same pass:
 *   cols_mode 0: dst[c][r * rows + i][k]   = src[r][c][i][k], k < seg
 *                (the ranks' row blocks stacked; dst_ld >= seg)
 *   cols_mode 1: dst[c][i][r * seg + k]    = src[r][c][i][k], k < seg
 *                (the ranks' k blocks concatenated; dst_ld >= world * seg)
 * seg, src_ld and dst_ld are multiples of 4. No reference counterpart. */
int fpb_trimul_group_gather(const void* src, int world, int channels, int rows, int src_ld,
                            int seg, int cols_mode, void* dst_hi, void* dst_lo, int dst_ld,
                            int precision, cudaStream_t stream);
int fpb_trimul_shard_finish(float* z_loc, int n, int rows, const void* x_blocked,
                            const float* ln_in_w, const float* ln_in_b, const float* w_g,
                            const float* ln_out_w, const float* ln_out_b, const float* w_z,
                            float eps, int add, int precision, void* workspace,
                            size_t workspace_bytes, cudaStream_t stream);
/* Triangle attention, starting-node form on the rank's rows: proj writes the
 * rank's q/k/v and gate (LayerNorm and all four projections, so it takes
 * w_g and b_g) and its rows of the pair bias; the caller all-gathers the
 * bias; finish runs the attention core (gate applied to o) and the output
 * projection on the rows (z_loc += delta, or delta_out = delta). The ending
 * node is this form on the transposed pair tensor (all-to-all transposes
 * around it). proj and finish share the workspace. The bias buffer is row-blocked: for ldb =
 * fpb_triattn_bias_ld(n), rows are grouped by 32, and rows [32q, 32q + 32m)
 * occupy the m*32*4*ldb floats starting at float q*32*4*ldb (so a rank whose
 * r0 and row chunk are multiples of 32 owns one contiguous range); the
 * buffer holds ceil(n/32)*32*4*ldb floats. */
size_t fpb_triattn_bias_ld(int n);
size_t fpb_triattn_shard_workspace_size(int n, int rows, int precision, int with_mask);
int fpb_triattn_shard_proj(const float* z_loc, const float* mask, int n, int rows, int r0,
                           const float* ln_w, const float* ln_b, const float* w_q,
                           const float* w_k, const float* w_v, const float* w_bias,
                           const float* w_g, const float* b_g, float eps, float* bias_full,
                           int precision, void* workspace, size_t workspace_bytes,
                           cudaStream_t stream);
int fpb_triattn_shard_finish(float* z_loc, float* delta_out, int n, int rows, int with_mask,
                             const float* bias_full, const float* w_o, const float* b_o,
                             int precision, void* workspace, size_t workspace_bytes,
                             cudaStream_t stream);

/* Peer memory for the row-sharded phases on the GPUs of one node (one
 * process per GPU). No reference counterpart (the reference has no sharded
 * path). fpb_ipc_export turns a device pointer of the caller's into a CUDA
 * IPC handle (fpb_ipc_handle_bytes bytes) of its allocation plus the
 * pointer's offset in it; another process maps it into its current device's
 * context with fpb_ipc_import (peer access enabled lazily; ptr_out = mapped
 * base + offset) and unmaps it with fpb_ipc_close(base). fpb_copy_async
 * enqueues one copy on `stream` (either pointer may be a mapped peer
 * address). The caller orders the copies against the owner's use of the
 * buffer (e.g. a collective on both sides). Nothing is allocated. */
size_t fpb_ipc_handle_bytes(void);
int fpb_ipc_export(const void* ptr, void* handle_out, size_t* offset_out);
int fpb_ipc_import(const void* handle, size_t offset, void** base_out, void** ptr_out);
int fpb_ipc_close(void* base);
int fpb_copy_async(void* dst, const void* src, size_t bytes, cudaStream_t stream);

/* Transposed exchange of the row-sharded pair tensor: rank `rank` of `world`
 * (world <= 16) owns rows [rank*chunk, rank*chunk + chunk) of z [n, n, ch]
 * as z_loc [chunk][n][ch] (rows at or past n are padding and are not read).
 * ch counts 4-byte words per pair (128 for FP32 c_z = 128); the kernel only
 * moves bytes, so any element type whose pair vector is ch words works.
 * Every owned z[i, j, :] with j < n is stored at row j - d*chunk, column i
 * of dst[d], d = j / chunk: dst[d] is rank d's [chunk][n][ch] buffer of the
 * rows of z^T it owns (a peer mapping, or the caller's own buffer for
 * d == rank). Rows of dst past n are not written. ch % 4 == 0, every pointer
 * 16-byte aligned. One kernel; the stores to other ranks cross NVLink. */
/* Up to 16 copies in one kernel: bytes[k] from src[k] to dst[k] (either
 * may be a mapped peer address), every pointer 16-byte aligned and every
 * size a multiple of 16 (zero sizes are skipped). The SMs issue the loads and
 * stores, so the copies to several peers cross NVLink side by side. The
 * caller orders them against the owners' use of the buffers. */
int fpb_peer_scatter(const void* const* src, void* const* dst, const size_t* bytes, int count,
                     cudaStream_t stream);

int fpb_peer_transpose_rows(const float* z_loc, int n, int chunk, int ch, int rank, int world,
                            float* const* dst, cudaStream_t stream);

/* Weights of the five pair operators of one block (torch Linear layouts). */
typedef struct {
  const float *ln_in_w, *ln_in_b, *w_a_p, *w_a_g, *w_b_p, *w_b_g, *w_g, *ln_out_w, *ln_out_b,
      *w_z;
} fpb_trimul_weights;
typedef struct {
  const float *ln_w, *ln_b, *w_q, *w_k, *w_v, *w_bias, *w_g, *b_g, *w_o, *b_o;
} fpb_triattn_weights;
typedef struct {
  const float *ln_w, *ln_b, *w_a, *w_b, *w_out;
} fpb_transition_weights;
typedef struct {
  fpb_trimul_weights tri_mul_out, tri_mul_in;
  fpb_triattn_weights tri_att_start, tri_att_end;
  fpb_transition_weights transition;
} fpb_pair_block_weights;

/* Pair stack of one Pairformer block, in place on z [n, n, 128]:
 * TriMul outgoing, TriMul incoming, TriAttn starting node, TriAttn ending
 * node, pair transition, each z += update (Protenix PairformerBlock with the
 * fireprot kernels, patches/protenix/0006-...patch:14-37). One workspace and
 * one status word for the whole block. */
size_t fpb_pair_block_workspace_size(int n, int precision, int with_mask);
int fpb_pair_block(float* z, const float* mask, int n, const fpb_pair_block_weights* weights,
                   float eps, int precision, void* workspace, size_t workspace_bytes,
                   cudaStream_t stream);

/* Weights of the single stack of one block (torch Linear layouts, c_s = 384,
 * 16 heads of 24): AttentionPairBias (layer_norm_a, linear_q with bias,
 * bias-free linear_k/v/g/o, layer_norm_z + bias-free linear_z to 16 heads)
 * and the single Transition (n = 4). */
typedef struct {
  const float *ln_a_w, *ln_a_b, *w_q, *b_q, *w_k, *w_v, *w_g, *w_o, *ln_z_w, *ln_z_b, *w_z;
  const float *tr_ln_w, *tr_ln_b, *tr_w_a, *tr_w_b, *tr_w_out;
} fpb_single_block_weights;

/* Single stack of one Pairformer block on query rows [r0, r0 + rows) of
 * s [n, 384] (in place): s += AttentionPairBias(s, z), then
 * s += Transition(s) (AlphaFold 3 Algorithms 24 without conditioning and 11).
 * z_loc holds pair rows [r0, r0 + rows) ([rows, n, 128]); mask is the full
 * [n, n] pair mask (nullable). Every row of s is read (keys and values), so a
 * row-sharded caller passes the whole s and all-gathers the rows afterwards;
 * an unsharded caller passes rows = n, r0 = 0.
 * No reference kernel: the reference runs this stack natively
 * (docs/openfold3-performance.md:68-74, "Single attention with pair bias",
 * "Single transition"). Runs in FP32 on CUDA cores in both precision modes
 * (`precision` is validated, the result is the same). */
size_t fpb_single_block_workspace_size(int n, int rows, int c_s);
int fpb_single_block(float* s, const float* z_loc, const float* mask, int n, int rows, int r0,
                     int c_s, const fpb_single_block_weights* weights, float eps, int precision,
                     void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* Triangle contraction on channels-last tensors, ESMFold2's form
 * (TriangleMultiplicativeBlock._triangular_contract_chunked as dispatched by
 * python/fireprot/adapters/esmfold2/triangle.py:19-33, C = 256 there):
 *   outgoing (outgoing = 1): out[i][j][c] = sum_k left[i][k][c] * right[j][k][c]
 *   incoming (outgoing = 0): out[i][j][c] = sum_k left[k][i][c] * right[k][j][c]
 * left, right, out: [n, n, channels] FP32, channels a multiple of 32. The
 * reference's chunking over i (chunk_size 64) only bounds its memory and is
 * not part of the result. */
size_t fpb_triangle_contract_workspace_size(int n, int channels, int precision);
int fpb_triangle_contract(const float* left, const float* right, float* out, int n, int channels,
                          int outgoing, int precision, void* workspace, size_t workspace_bytes,
                          cudaStream_t stream);

/* Per-launch device timing on the calling thread (CUDA events around every
 * kernel launch of this library). fpb_timing_collect synchronises and writes
 * {"kernel": {"launches": L, "total_ms": T}, ...} as JSON. */
int fpb_timing_enable(int on);
int fpb_timing_collect(char* out, size_t cap);

#ifdef __cplusplus
}
#endif

#endif /* FIREPROT_B200_H */
