// gemm_fp16 section of the shipped launch.cu: tempo::gen::launch / plan for GemmParams.  The
// dispatch body is the generated dispatch.inc (the reference's launch.cu:20-22 shape): a table
// of M-ladder rows, the first row covering M picks the hyperform family, and a problem no row
// covers returns cudaErrorInvalidConfiguration.
namespace tempo_sm100 {
namespace {

// One ladder row applied to an fp16 problem: plan it (plan_only != nullptr) or launch it.
cudaError_t fp16_by_row(const tempo::gen::GemmParams& p, const LadderRow& row, cudaStream_t s,
                        tempo::gen::Choice* plan_only) {
  const int sms = current_sms();
  // a plan is made for the workspace size it is given; a launch only has a workspace if ws
  // is non-NULL
  const size_t cap = plan_only ? p.ws_bytes : (p.ws ? p.ws_bytes : 0);
  Hyper h{};
  if (!select_hyper(0, row, p.M, p.N, p.K, cap, h, sms)) return cudaErrorInvalidConfiguration;
  if (plan_only) {
    tempo::gen::Choice& c = *plan_only;
    c.bn = h.bn;
    c.swap = h.swap;
    c.splits = h.splits;
    c.group_m = h.group_m;
    c.cta_group = h.cta_group;
    c.expand = 0;
    const InstEntry* e = h.cta_group == 1 ? find_inst(0, h.bn, h.swap) : nullptr;
    c.stages = e ? e->stages : 0;
    c.ws_bytes = hyper_ws(p.M, p.N, p.K, h, sms, cap, &c.zero_bytes);
    return cudaSuccess;
  }
  const Problem pr{0, p.A, p.B, nullptr, nullptr, p.C, p.M, p.N, p.K, p.lda, p.ldb, p.ldc,
                   0, p.ws, p.ws_bytes};
  return run(pr, h, s);
}

}  // namespace
}  // namespace tempo_sm100

namespace tempo {
namespace gen {
namespace {

cudaError_t dispatch_gemm_fp16(const GemmParams& p, cudaStream_t s, Choice* plan_only) {
  using tempo_sm100::LadderRow;
  using tempo_sm100::fp16_by_row;
#include "dispatch.inc"
}

}  // namespace

cudaError_t launch(const GemmParams& p, cudaStream_t s) {
  if (!applicable(p)) return cudaErrorInvalidConfiguration;
  if (p.ws && !tempo_sm100::aligned16(p.ws)) return cudaErrorInvalidValue;
  return dispatch_gemm_fp16(p, s, nullptr);
}

cudaError_t plan(const GemmParams& p, Choice* out) {
  if (!shape_ok(p) || !out) return cudaErrorInvalidConfiguration;
  *out = Choice{};
  return dispatch_gemm_fp16(p, nullptr, out);
}

}  // namespace gen
}  // namespace tempo
