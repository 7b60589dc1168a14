// Program optimiser: pattern rewrites over a recorded window.
//
// The typed executor (include/passes/execute.h, JTPuffer/TempLit) emits one
// runtime call per expression node, so fusable work reaches the runtime as
// short op sequences.  Because the runtime records a whole window before it
// launches anything, it can see those sequences and replace them with one
// kernel, provided every value another op (or the host, after wait()) can
// still observe comes out identical.  Intermediates are only skipped when
// their storage is released inside the window and nothing else reads them.
#include "optimize.h"

#include <algorithm>
#include <unordered_map>
#include <unordered_set>

namespace cuda::internal {
namespace {

bool is_opt(Kind k) {
  return k == Kind::SqNorm || k == Kind::Clip || k == Kind::AdamW;
}

// `Compiled::step(max_norm)` (include/passes/compile.h:236-258) records
//   SqNorm(g_i, n) for every gradient, Clip(g_i, n, c, g_i) for every
//   gradient, then AdamW(p_i, g_i, p_i, m1_i, m2_i, b1, b2, decay, lr, eps, t_i)
// and `Compiled::step()` records the AdamW calls alone.  Both become one
// MultiAdamW op (two launches: deterministic norm, then clip + update).
uint64_t fuse_step(std::vector<Op> &p) {
  std::vector<size_t> norms, clips, adams;
  size_t first = p.size(), last = 0;
  for (size_t i = 0; i < p.size(); ++i) {
    const Op &op = p[i];
    if (op.dead) continue;
    if (op.kind == Kind::SqNorm) norms.push_back(i);
    else if (op.kind == Kind::Clip) clips.push_back(i);
    else if (op.kind == Kind::AdamW) adams.push_back(i);
    else continue;
    first = std::min(first, i);
    last = std::max(last, i);
  }
  if (adams.empty()) return 0;
  // strict phase order and nothing but storage initialisation in between
  if (!norms.empty() && (clips.empty() || norms.back() > clips.front())) return 0;
  if (!clips.empty() && clips.back() > adams.front()) return 0;
  if (norms.empty() != clips.empty()) return 0;
  for (size_t i = first; i <= last; ++i) {
    const Op &op = p[i];
    if (op.dead || is_opt(op.kind)) continue;
    if (op.kind != Kind::Fill && op.kind != Kind::Release) return 0;
  }
  const Op &a0 = p[adams.front()];
  std::unordered_set<void *> grads;
  for (size_t i : adams) {
    const Op &op = p[i];
    for (int j = 5; j <= 8; ++j)
      if (op.t[j].p != a0.t[j].p) return 0;
    if (op.f0 != a0.f0) return 0;
    if (!grads.insert(op.t[1].p).second) return 0;  // each gradient updated once
  }
  void *sq = nullptr;
  float max_norm = 0.0f;
  if (!clips.empty()) {
    sq = p[norms.front()].t[1].p;
    max_norm = p[clips.front()].f0;
    std::unordered_set<void *> normed, clipped;
    for (size_t i : norms) {
      if (p[i].t[1].p != sq || !normed.insert(p[i].t[0].p).second) return 0;
    }
    for (size_t i : clips) {
      const Op &op = p[i];
      if (op.t[1].p != sq || op.f0 != max_norm || op.t[0].p != op.t[2].p) return 0;
      if (!clipped.insert(op.t[0].p).second) return 0;
    }
    if (normed != grads || clipped != grads) return 0;
  }
  Op fused;
  fused.kind = Kind::MultiAdamW;
  if (sq) fused.t[0] = p[norms.front()].t[1];
  for (int j = 5; j <= 8; ++j) fused.t[j] = a0.t[j];
  fused.f0 = max_norm;
  fused.f1 = a0.f0;
  uint64_t chunks = 0;
  for (size_t i : adams) {
    const Op &op = p[i];
    MultiSlot s;
    s.param = op.t[0];
    s.grad = op.t[1];
    s.out = op.t[2];
    s.m1 = op.t[3];
    s.m2 = op.t[4];
    s.step = op.u0;
    chunks += (op.t[0].numel() + TL_OPT_CHUNK - 1) / TL_OPT_CHUNK;
    fused.multi.push_back(s);
  }
  fused.workspace = tl_multi_clip_adamw_workspace_size(static_cast<uint32_t>(chunks));
  const uint64_t folded = norms.size() + clips.size() + adams.size() - 1;
  for (size_t i : norms) p[i].dead = true;
  for (size_t i : clips) p[i].dead = true;
  for (size_t i : adams) p[i].dead = true;
  p[adams.back()] = std::move(fused);
  return folded;
}

}  // namespace

void add_gradient_allreduce(std::vector<Op> &prog) {
  size_t first = prog.size();
  Op ar;
  ar.kind = Kind::AllReduce;
  std::unordered_set<void *> seen;
  for (size_t i = 0; i < prog.size(); ++i) {
    const Op &op = prog[i];
    if (op.dead) continue;
    const bool opt = op.kind == Kind::SqNorm || op.kind == Kind::Clip ||
                     op.kind == Kind::AdamW || op.kind == Kind::MultiAdamW;
    if (!opt) continue;
    first = std::min(first, i);
    if (op.kind == Kind::AdamW && seen.insert(op.t[1].p).second) {
      MultiSlot s{};
      s.grad = op.t[1];
      ar.multi.push_back(s);
    }
    if (op.kind == Kind::MultiAdamW)
      for (const MultiSlot &m : op.multi)
        if (seen.insert(m.grad.p).second) {
          MultiSlot s{};
          s.grad = m.grad;
          ar.multi.push_back(s);
        }
  }
  if (ar.multi.empty()) return;
  prog.insert(prog.begin() + static_cast<std::ptrdiff_t>(first), std::move(ar));
}

uint64_t optimize(std::vector<Op> &prog, void *comm) {
  uint64_t folded = 0;
  folded += fuse_step(prog);
  if (comm) add_gradient_allreduce(prog);
  return folded;
}

}  // namespace cuda::internal
