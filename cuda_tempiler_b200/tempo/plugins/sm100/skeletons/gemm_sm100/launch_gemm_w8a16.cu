// gemm_w8a16 section of the shipped launch.cu: tempo::gen::launch / plan for W8A16Params.  The
// dispatch body is the generated dispatch.inc: the prefill expansion (from a generated M, when
// the workspace holds the fp16 copy), then the M-ladder rows of the in-kernel dequant tiles and
// the decode GEMV; a problem nothing covers returns cudaErrorInvalidConfiguration.
namespace tempo_sm100 {
namespace {

Problem w8_problem(const tempo::gen::W8A16Params& p) {
  return Problem{p.scale_kind, p.A, p.W, p.scale, p.zero, p.C, p.M, p.N, p.K,
                 p.lda, p.ldw, p.ldc, p.group, p.ws, p.ws_bytes};
}

void fill_choice(tempo::gen::Choice& c, const Hyper& h, int wkind) {
  c.bn = h.bn;
  c.swap = h.swap;
  c.splits = h.splits;
  c.group_m = h.group_m;
  c.cta_group = h.cta_group;
  const InstEntry* e = h.cta_group == 1 ? find_inst(wkind, h.bn, h.swap) : nullptr;
  c.stages = e ? e->stages : 0;
}

// Prefill: expand the 8-bit weights to fp16 in the workspace (after its counter prefix), then
// run the fp16 hyperform of `row` on the copy, its partials after the copy.  *taken is false
// (nothing planned or launched) when the workspace cannot hold the copy or the row does not
// apply.
cudaError_t w8_expanded(const tempo::gen::W8A16Params& p, const LadderRow& row, cudaStream_t s,
                        tempo::gen::Choice* plan_only, bool* taken) {
  *taken = false;
  const size_t cap = plan_only ? p.ws_bytes : (p.ws ? p.ws_bytes : 0);
  const size_t wexp = expand_ws_bytes(p.N, p.K);
  // layout: [counter prefix | fp16 weights (wexp) | fp32 partials of the fp16 launch]
  if (cap < kExpandOffset + wexp) return cudaSuccess;
  const int sms = current_sms();
  Hyper h{};
  if (!select_hyper(0, row, p.M, p.N, p.K, cap - wexp, h, sms)) return cudaSuccess;
  *taken = true;
  if (plan_only) {
    fill_choice(*plan_only, h, 0);
    plan_only->expand = 1;
    size_t zero = 0;
    const size_t need = hyper_ws(p.M, p.N, p.K, h, sms, cap - wexp, &zero);
    plan_only->ws_bytes = kExpandOffset + wexp + (need > kCounterBytes ? need - kCounterBytes : 0);
    plan_only->zero_bytes = zero;
    return cudaSuccess;
  }
  char* base = static_cast<char*>(p.ws);
  __half* wf = reinterpret_cast<__half*>(base + kExpandOffset);
  const cudaError_t e = launch_expand(w8_problem(p), wf, s);
  if (e != cudaSuccess) return e;
  Problem pr{0, p.A, wf, nullptr, nullptr, p.C, p.M, p.N, p.K, p.lda, p.K, p.ldc, 0,
             p.ws, p.ws_bytes - wexp};
  pr.ws_parts = base + kExpandOffset + wexp;
  return run(pr, h, s);
}

// One ladder row with the weights dequantised inside the kernel (tiles or the GEMV).
cudaError_t w8_by_row(const tempo::gen::W8A16Params& p, const LadderRow& row, cudaStream_t s,
                      tempo::gen::Choice* plan_only) {
  const int sms = current_sms();
  const size_t cap = plan_only ? p.ws_bytes : (p.ws ? p.ws_bytes : 0);
  Hyper h{};
  if (!select_hyper(p.scale_kind, row, p.M, p.N, p.K, cap, h, sms))
    return cudaErrorInvalidConfiguration;
  if (plan_only) {
    fill_choice(*plan_only, h, p.scale_kind);
    plan_only->expand = 0;
    plan_only->ws_bytes = hyper_ws(p.M, p.N, p.K, h, sms, cap, &plan_only->zero_bytes);
    return cudaSuccess;
  }
  return run(w8_problem(p), h, s);
}

}  // namespace
}  // namespace tempo_sm100

namespace tempo {
namespace gen {
namespace {

cudaError_t dispatch_gemm_w8a16(const W8A16Params& p, cudaStream_t s, Choice* plan_only) {
  using tempo_sm100::LadderRow;
  using tempo_sm100::w8_by_row;
  using tempo_sm100::w8_expanded;
#include "dispatch.inc"
}

}  // namespace

cudaError_t launch(const W8A16Params& p, cudaStream_t s) {
  if (!applicable(p)) return cudaErrorInvalidConfiguration;
  // the expanded weights are written with 16-byte stores from the start of ws
  if (p.ws && !tempo_sm100::aligned16(p.ws)) return cudaErrorInvalidValue;
  return dispatch_gemm_w8a16(p, s, nullptr);
}

cudaError_t plan(const W8A16Params& p, Choice* out) {
  if (!shape_ok(p) || !out) return cudaErrorInvalidConfiguration;
  *out = Choice{};
  return dispatch_gemm_w8a16(p, nullptr, out);
}

}  // namespace gen
}  // namespace tempo
