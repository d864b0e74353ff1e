// Pair stack of one Pairformer block on one stream:
//   TriMul outgoing, TriMul incoming, TriAttn starting node, TriAttn ending
//   node, pair transition, each adding its update to z in place
// (order of patches/protenix/0006-...patch:14-37, AF3 Algorithm 17).
// One workspace is shared by the five operators (they run back to back on
// the same stream); its status word covers the whole block.
#include "kernels.h"
#include "../../include/fireprot_b200.h"

namespace fpb {

namespace {
thread_local int g_composite_depth = 0;
}

CompositeCall::CompositeCall() { ++g_composite_depth; }
CompositeCall::~CompositeCall() { --g_composite_depth; }

int sm_count() {
  static int cached[64] = {0};  // benign race: every writer stores the same value
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int c = 0;
    if (cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || c <= 0)
      c = 148;
    cached[dev] = c;
  }
  return cached[dev];
}

int reset_status(void* workspace, cudaStream_t stream) {
  if (g_composite_depth > 0) return kOk;
  return cudaMemsetAsync(workspace, 0, kWsHeader, stream) == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace fpb

using namespace fpb;

extern "C" size_t fpb_pair_block_workspace_size(int n, int precision, int with_mask) {
  const size_t a = fpb_trimul_workspace_size(n, 128, precision);
  const size_t b = fpb_triattn_workspace_size(n, 128, 4, 32, precision, with_mask);
  const size_t c = fpb_transition_workspace_size(128, 4, precision);
  if (!a || !b || !c) return 0;
  size_t m = a > b ? a : b;
  return m > c ? m : c;
}

extern "C" int fpb_pair_block(float* z, const float* mask, int n,
                              const fpb_pair_block_weights* w, float eps, int precision,
                              void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!w || !z || !workspace) return kErrArg;
  const size_t need = fpb_pair_block_workspace_size(n, precision, mask != nullptr);
  if (!need) return kErrShape;
  if (workspace_bytes < need) return kErrWorkspace;
  if (!aligned16(workspace)) return kErrAlign;
  if (cudaMemsetAsync(workspace, 0, kWsHeader, stream) != cudaSuccess) return kErrCuda;
  CompositeCall scope;
  int st;
  const fpb_trimul_weights* tm[2] = {&w->tri_mul_out, &w->tri_mul_in};
  for (int d = 0; d < 2; ++d) {
    const fpb_trimul_weights& t = *tm[d];
    st = fpb_trimul(z, mask, n, 128, t.ln_in_w, t.ln_in_b, t.w_a_p, t.w_a_g, t.w_b_p, t.w_b_g,
                    t.w_g, t.ln_out_w, t.ln_out_b, t.w_z, eps, d == 0 ? 1 : 0, 1, precision,
                    workspace, workspace_bytes, stream);
    if (st) return st;
  }
  const fpb_triattn_weights* ta[2] = {&w->tri_att_start, &w->tri_att_end};
  for (int d = 0; d < 2; ++d) {
    const fpb_triattn_weights& a = *ta[d];
    st = fpb_triattn(z, nullptr, mask, n, 128, 4, 32, a.ln_w, a.ln_b, a.w_q, a.w_k, a.w_v, a.w_bias, a.w_g,
                     a.b_g, a.w_o, a.b_o, eps, d == 0 ? 1 : 0, precision, workspace,
                     workspace_bytes, stream);
    if (st) return st;
  }
  const fpb_transition_weights& tr = w->transition;
  return fpb_transition(z, nullptr, (long long)n * n, 128, 4, tr.ln_w, tr.ln_b, tr.w_a, tr.w_b, tr.w_out,
                        eps, precision, workspace, workspace_bytes, stream);
}
