// cuda::Runtime: argument validation and recording of every runtime call,
// program execution (eager or CUDA-graph replay) and the window lifecycle.
//
// Each op method mirrors the corresponding metal::Runtime method of
// JTPuffer/TempLit (src/my_metal/runtime.cpp, cited per method): it throws
// the same exception type with the same text on the same bad arguments
// (with "CUDA" in place of "Metal"), then appends one Op to the window.
#include "my_cuda/runtime.h"

#include "RTensor/dimension.h"
#include "RTensor/infer_shape.h"
#include "optimize.h"
#include "program.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <map>
#include <numeric>
#include <stdexcept>
#include <unordered_map>
#include <unordered_set>

namespace cuda {

using internal::check;
using internal::Kind;
using internal::Op;
using internal::TRef;

namespace {

using Mat = RTensor<CUDA, kernel_type>;
using IndexMat = RTensor<CUDA, index_type>;

template <typename T>
TRef ref(const RTensor<CUDA, T> &m) {
  TRef r;
  const Storage<CUDA, T> *s = m.get_storage();
  if (!s) throw std::logic_error("runtime op on an uninitialised tensor");
  if (m.shape().size() > static_cast<size_t>(internal::kMaxRank))
    throw std::invalid_argument("tensor rank exceeds the CUDA runtime limit of 8");
  r.p = const_cast<T *>(s->data());
  r.id = s->block().id;
  r.rank = static_cast<uint8_t>(m.shape().size());
  for (size_t i = 0; i < m.shape().size(); ++i) r.shape[i] = m.shape()[i];
  return r;
}

TRef ref_block(const detail::Block &b, uint64_t bytes) {
  TRef r;
  r.p = b.ptr;
  r.id = b.id;
  r.rank = 1;
  r.shape[0] = static_cast<uint32_t>(bytes);
  return r;
}

// Broadcast check of an operand against the destination shape
// (src/my_metal/runtime.cpp:18-39).
void check_broadcast(std::span<const uint32_t> shape, std::span<const uint32_t> out) {
  if (shape.size() > out.size()) throw std::runtime_error("invalid broadcast");
  const size_t off = out.size() - shape.size();
  for (size_t i = 0; i < shape.size(); ++i)
    if (shape[i] != out[off + i] && shape[i] != 1) throw std::runtime_error("invalid broadcast");
}

const char *const kKindNames[] = {
    "binary",  "scalar",    "unary",      "copy",       "reduce",    "argmax",   "transpose",
    "softmax", "rms",       "rmsnorm",    "xent",       "xent_bwd",  "gather",   "scatter",
    "sqnorm",  "clip",      "adamw",      "gemm",       "host_write", "fill",    "dev_copy",
    "release", "gelu_bwd",  "softmax_bwd", "rmsnorm_bwd", "multi_adamw", "allreduce",
    "attention", "flash_fwd", "flash_bwd", "flash_probs"};

}  // namespace

namespace internal {
const char *kind_name(Kind k) { return kKindNames[static_cast<int>(k)]; }
}  // namespace internal

// ---------------------------------------------------------------------------
struct Runtime::Impl : internal::Recorder, internal::Liveness, internal::FlashState,
                       internal::HostAccessHook {
  enum class State { Idle, Recording, Submitted };
  State state = State::Idle;
  uint64_t window_id = 0;
  std::vector<Op> prog;
  RuntimeStats stats;
  bool fusion = true;
  bool graphs = true;
  int gemm_precision = TL_GEMM_TF32;
  void *comm = nullptr;

  // flash attention: P tensors left virtual by launched programs, their
  // log-sum-exp buffers, and one causal-check word per mask allocation
  // 0 off, 1 where the short-sequence fused kernels cannot run (T > 192;
  // they are faster up to there), 2 always; TL_FLASH_ATTENTION overrides
  int flash = [] {
    const char *e = std::getenv("TL_FLASH_ATTENTION");
    return e ? std::atoi(e) : 1;
  }();
  std::vector<internal::FlashRecord> flash_records;
  std::unordered_map<uint64_t, detail::Block> lse_blocks, mask_words;

  bool enabled() const override { return flash != 0; }
  bool always() const override { return flash >= 2; }
  const std::vector<internal::FlashRecord> &records() const override { return flash_records; }
  float *lse_buffer(uint64_t p_id, size_t bytes) override {
    auto it = lse_blocks.find(p_id);
    if (it != lse_blocks.end() && it->second.bytes >= bytes) return static_cast<float *>(it->second.ptr);
    if (it != lse_blocks.end()) detail::release(it->second);
    detail::Block b = detail::allocate(bytes);
    lse_blocks[p_id] = b;
    return static_cast<float *>(b.ptr);
  }
  uint32_t *mask_word(uint64_t mask_id) override {
    auto it = mask_words.find(mask_id);
    if (it == mask_words.end()) it = mask_words.emplace(mask_id, detail::allocate(16)).first;
    return static_cast<uint32_t *>(it->second.ptr);
  }
  // P of `f` from its recipe, now, on the runtime's stream
  void materialise(const internal::FlashRecord &f) {
    check(tl_flash_attention_probs(&f.desc, f.p.f(), cuda::stream()), "flash attention P");
    ++stats.flash_rebuilt;
  }
  void before_host_access(uint64_t id, bool write, bool full) override {
    for (size_t r = 0; r < flash_records.size();) {
      internal::FlashRecord &f = flash_records[r];
      const bool recipe = id == f.q.id || id == f.k.id || id == f.divisor.id ||
                          (f.mask.p && id == f.mask.id);
      if ((id == f.p_id && !(write && full)) || (write && recipe)) materialise(f);
      if (id == f.p_id || (write && recipe)) {
        flash_records.erase(flash_records.begin() + static_cast<std::ptrdiff_t>(r));
        continue;
      }
      if (write && id == f.o.id) f.o_valid = false;
      ++r;
    }
  }
  void on_release(uint64_t id) noexcept override {
    for (size_t r = 0; r < flash_records.size();) {
      const internal::FlashRecord &f = flash_records[r];
      const bool recipe = id == f.q.id || id == f.k.id || id == f.divisor.id ||
                          (f.mask.p && id == f.mask.id);
      if (recipe && cuda::initialised()) {
        try {
          materialise(f);  // its input is about to go
        } catch (...) {
        }
      }
      if (id == f.p_id || recipe) {
        flash_records.erase(flash_records.begin() + static_cast<std::ptrdiff_t>(r));
        continue;
      }
      ++r;
    }
    auto it = lse_blocks.find(id);
    if (it != lse_blocks.end()) {
      const detail::Block b = it->second;
      lse_blocks.erase(it);
      detail::release(b);
    }
    auto mw = mask_words.find(id);
    if (mw != mask_words.end()) {
      const detail::Block b = mw->second;
      mask_words.erase(mw);
      detail::release(b);
    }
  }

  // scratch shared by the ops of a program (they run one after another)
  detail::Block workspace;
  // fused optimiser slot tables: device copy + pinned host staging
  detail::Block slot_dev;
  void *slot_host = nullptr;
  size_t slot_capacity = 0;
  // gradients packed for the data-parallel all-reduce (one NCCL call)
  detail::Block flat_dev;

  // graph cache: program signature -> instantiated graph
  struct Cached {
    void *exec = nullptr;
    uint64_t kernels = 0;
    uint64_t last_use = 0;
  };
  std::unordered_map<std::string, Cached> graph_cache;
  // programs seen once (forward, backward and step windows alternate, so a
  // program recurs every few windows); captured on the second sighting
  std::unordered_map<std::string, uint64_t> seen_once;
  uint64_t use_clock = 0;

  // profiling
  bool profiling = false;
  std::string profile_path;
  struct Prof {
    uint64_t calls = 0;
    double ms = 0.0;
    double bytes = 0.0;  // algorithmic HBM bytes of the memory-bound ops
  };
  std::map<std::string, Prof> profile;

  // window liveness: per allocation, whether some recorded program read it
  // before writing it (its value crosses windows) and how many programs
  // opened by fully overwriting it
  struct Life {
    bool crossed = false;
    uint32_t fresh_writes = 0;
  };
  std::unordered_map<uint64_t, Life> life;
  uint64_t optimizer_windows = 0;

  // program listings (TL_PROGRAM_DUMP=<file>): each distinct recorded
  // program once, as recorded and as optimised
  std::string dump_path = [] {
    const char *e = std::getenv("TL_PROGRAM_DUMP");
    return std::string(e ? e : "");
  }();
  std::unordered_set<std::string> dumped;

  // host timing per window (TL_HOST_TRACE=<file>): recorded ops, host ns
  // recording, optimising, launching; written when the runtime is destroyed
  std::string trace_path = [] {
    const char *e = std::getenv("TL_HOST_TRACE");
    return std::string(e ? e : "");
  }();
  struct WindowTime {
    uint64_t ops, record_ns, optimise_ns, launch_ns;
  };
  std::vector<WindowTime> trace;

  void write_trace() {
    if (trace_path.empty() || trace.empty()) return;
    std::ofstream out(trace_path);
    out << "ops,record_us,optimise_us,launch_us\n";
    for (const auto &w : trace)
      out << w.ops << "," << w.record_ns / 1000.0 << "," << w.optimise_ns / 1000.0 << ","
          << w.launch_ns / 1000.0 << "\n";
    trace.clear();
  }

  // Optimised programs by recorded-program signature.  A training loop
  // records the same few programs every step; their optimised form is
  // reused while every buffer the optimiser relied on as window-local still
  // is.  Only Storage write payloads vary between recordings of one
  // signature, and they are copied from the new recording.
  struct Plan {
    std::vector<Op> ops;
    std::vector<uint64_t> local_ids;  // window_local() answers that were true
    uint64_t folded = 0;
    uint64_t last_use = 0;
    std::string graph_sig;  // signature of the optimised program
  };
  const std::string *planned_sig = nullptr;  // this submit's, when cached
  std::unordered_map<std::string, Plan> plans;

  // deferred wait: this window's status word is moved to pinned memory in
  // stream order and read by a later wait() once its event has passed
  bool deferred_wait = false;
  uint32_t *status_host = nullptr;
  void *status_event = nullptr;
  bool status_pending = false;
  std::chrono::steady_clock::time_point record_t0;

  // Liveness view that remembers which buffers it reported window-local.
  struct NotingLiveness : internal::Liveness {
    const Impl *impl;
    mutable std::vector<uint64_t> yes;
    explicit NotingLiveness(const Impl *i) : impl(i) {}
    bool window_local(uint64_t id) const override {
      const bool v = impl->window_local(id);
      if (v) yes.push_back(id);
      return v;
    }
  };

  void optimise_program() {
    observe(prog);
    std::string key = signature(prog);
    key += optimizer_windows >= 2 ? 'L' : '-';
    key += comm ? 'C' : '-';
    // the optimised form depends on which P tensors are virtual
    for (const internal::FlashRecord &f : flash_records) {
      key.append(reinterpret_cast<const char *>(&f.p_id), sizeof(f.p_id));
      key += f.o_valid ? 'o' : '-';
    }
    auto it = plans.find(key);
    if (it != plans.end()) {
      bool valid = true;
      for (uint64_t id : it->second.local_ids)
        if (!window_local(id)) {
          valid = false;
          break;
        }
      if (valid) {
        std::vector<Op> recorded = std::move(prog);
        prog = it->second.ops;
        for (Op &op : prog)
          if (op.kind == Kind::HostWrite && op.src < recorded.size())
            op.host = std::move(recorded[op.src].host);
        stats.fused_ops += it->second.folded;
        ++stats.optimiser_cache_hits;
        it->second.last_use = ++use_clock;
        planned_sig = &it->second.graph_sig;
        return;
      }
      plans.erase(it);
    }
    for (size_t i = 0; i < prog.size(); ++i) prog[i].src = static_cast<uint32_t>(i);
    NotingLiveness live(this);
    Plan plan;
    plan.folded = internal::optimize(prog, comm, &live, this);
    stats.fused_ops += plan.folded;
    // small programs re-optimise cheaply; optimiser-step programs carry the
    // step count in their signature and never recur
    if (prog.size() < 64) return;
    for (const Op &op : prog)
      if (op.kind == Kind::AdamW || op.kind == Kind::MultiAdamW) return;
    if (plans.size() >= 16) {
      auto victim = plans.begin();
      for (auto p = plans.begin(); p != plans.end(); ++p)
        if (p->second.last_use < victim->second.last_use) victim = p;
      plans.erase(victim);
    }
    plan.ops = prog;
    for (Op &op : plan.ops) op.host.clear();
    plan.local_ids = std::move(live.yes);
    plan.last_use = ++use_clock;
    plan.graph_sig = signature(prog);
    planned_sig = &plans.emplace(std::move(key), std::move(plan)).first->second.graph_sig;
  }

  ~Impl() override {
    write_trace();
    release_resources();
  }

  // One line per op; with `marks`, each tensor carries its liveness as the
  // optimiser saw it: '*' window-local, '^' read by the host.
  std::string describe(const Op &op, bool marks = false) const {
    std::string s = internal::kind_name(op.kind);
    if (op.kind == Kind::Binary || op.kind == Kind::Unary || op.kind == Kind::Scalar ||
        op.kind == Kind::Reduce)
      s += "#" + std::to_string(op.code);
    if (op.kind == Kind::Gemm) {
      const auto &g = op.gemm;
      s += " " + std::to_string(g.m) + "x" + std::to_string(g.n) + "x" + std::to_string(g.k);
      s += g.trans_a ? " T" : " N";
      s += g.trans_b ? "T" : "N";
      for (uint32_t i = 0; i < g.batch_rank; ++i)
        s += (i ? "," : " b[") + std::to_string(g.batch_shape[i]) + "/" +
             std::to_string(g.a_batch_stride[i]) + ":" + std::to_string(g.b_batch_stride[i]) +
             ":" + std::to_string(g.c_batch_stride[i]) + (i + 1 == g.batch_rank ? "]" : "");
      if (g.beta != 0.0f) s += " beta";
      if (g.bias) s += " bias";
      if (g.gelu_out) s += " gelu";
    }
    if (op.kind == Kind::Transpose) s += " " + std::to_string(op.i0) + "<>" + std::to_string(op.i1);
    if (op.kind == Kind::Scalar) s += " " + std::to_string(op.f0);
    for (int i = 0; i < 9; ++i) {
      const TRef &r = op.t[i];
      if (!r.p && !r.id) continue;
      s += " t" + std::to_string(i) + "=" + std::to_string(r.id) + "[";
      for (int d = 0; d < r.rank; ++d) s += (d ? "," : "") + std::to_string(r.shape[d]);
      s += "]";
      if (marks && r.id) {
        if (window_local(r.id)) s += "*";
        if (internal::host_observed(r.id)) s += "^";
      }
    }
    if (!op.multi.empty()) s += " slots=" + std::to_string(op.multi.size());
    if (op.dead) s += " DEAD";
    return s;
  }

  void dump(const char *title, bool fresh) {
    std::ofstream out(dump_path, std::ios::app);
    out << "== " << title << " window " << window_id << (fresh ? "" : " (again)") << " ops "
        << prog.size() << "\n";
    for (size_t i = 0; i < prog.size(); ++i) out << i << " " << describe(prog[i], true) << "\n";
  }

  // Updates `life` from a recorded (not yet optimised) program.
  void observe(const std::vector<Op> &p) {
    std::unordered_set<uint64_t> touched;
    bool updates = false;
    for (const Op &op : p) {
      if (op.kind == Kind::Release) {
        life.erase(op.t[0].id);
        continue;
      }
      if (op.kind == Kind::AdamW) updates = true;
      const internal::Access a = internal::access(op);
      for (int i = 0; i < a.nr; ++i)
        if (touched.insert(a.r[i]).second) life[a.r[i]].crossed = true;
      for (int i = 0; i < a.nw; ++i)
        if (touched.insert(a.w[i]).second) {
          Life &l = life[a.w[i]];
          if (internal::full_write(op)) ++l.fresh_writes;
          else l.crossed = true;
        }
    }
    if (updates) ++optimizer_windows;
  }

  // ---- Liveness: a buffer is window-local once two optimiser steps have
  // run, every program so far that touched it overwrote it first (at least
  // twice), and the host never read it.
  bool window_local(uint64_t id) const override {
    if (optimizer_windows < 2) return false;
    const auto it = life.find(id);
    return it != life.end() && !it->second.crossed && it->second.fresh_writes >= 2 &&
           !internal::host_observed(id);
  }

  // ---- Recorder
  uint64_t window() const override { return state == State::Recording ? window_id : 0; }
  void record_write(const detail::Block &dst, size_t offset, const void *src,
                    size_t bytes) override {
    Op &op = push(Kind::HostWrite);
    op.t[0] = ref_block(dst, dst.bytes);
    op.n = offset;
    op.host.assign(static_cast<const uint8_t *>(src), static_cast<const uint8_t *>(src) + bytes);
  }
  void record_fill(const detail::Block &dst, uint32_t pattern, size_t count) override {
    Op &op = push(Kind::Fill);
    op.t[0] = ref_block(dst, dst.bytes);
    op.u0 = pattern;
    op.n = count;
  }
  void record_copy(const detail::Block &dst, const detail::Block &src, size_t bytes) override {
    Op &op = push(Kind::DevCopy);
    op.t[0] = ref_block(dst, dst.bytes);
    op.t[1] = ref_block(src, src.bytes);
    op.n = bytes;
  }
  void record_release(const detail::Block &b) override {
    if (state != State::Recording) return;
    Op &op = push(Kind::Release);
    op.t[0].id = b.id;
    op.t[0].p = b.ptr;
    op.n = b.bytes;  // the address range the pool may hand out again
  }

  Op &push(Kind k) {
    prog.emplace_back();
    Op &op = prog.back();
    op.kind = k;
    return op;
  }

  Op &record(Kind k) {
    if (state != State::Recording)
      throw std::logic_error("CUDA runtime execution has not started");
    ++stats.ops_recorded;
    return push(k);
  }

  uint32_t deferred_status() {
    uint32_t flags = 0;
    if (!status_host) {
      void *p = nullptr;
      check(tl_host_alloc(&p, sizeof(uint32_t)), "status staging");
      status_host = static_cast<uint32_t *>(p);
      check(tl_event_create(&status_event), "status event");
    }
    if (status_pending) {
      int done = 0;
      check(tl_event_query(status_event, &done), "status event");
      if (done) {
        flags = *status_host;
        status_pending = false;
      }
    }
    if (!status_pending) {
      // flags raised since the last move stay in the device word until then
      check(tl_device_status_enqueue(status_host, cuda::stream()), "status");
      check(tl_event_record(status_event, cuda::stream()), "status event");
      status_pending = true;
    }
    return flags;
  }

  void release_resources() noexcept {
    for (auto &kv : graph_cache) tl_graph_destroy(kv.second.exec);
    flash_records.clear();
    for (auto *m : {&lse_blocks, &mask_words}) {
      std::vector<detail::Block> blocks;
      for (auto &kv : *m) blocks.push_back(kv.second);
      m->clear();
      for (const detail::Block &b : blocks) detail::release(b);
    }
    if (status_host) {
      if (cuda::initialised()) {
        tl_stream_sync(cuda::stream());
        tl_host_free(status_host);
        tl_event_destroy(status_event);
      }
      status_host = nullptr;
      status_event = nullptr;
      status_pending = false;
    }
    graph_cache.clear();
    seen_once.clear();
    if (workspace.ptr) {
      detail::release(workspace);
      workspace = detail::Block{};
    }
    if (slot_dev.ptr) {
      detail::release(slot_dev);
      slot_dev = detail::Block{};
    }
    if (slot_host) {
      tl_host_free(slot_host);
      slot_host = nullptr;
    }
    slot_capacity = 0;
    if (flat_dev.ptr) {
      detail::release(flat_dev);
      flat_dev = detail::Block{};
    }
  }

  // ---- execution
  void ensure_workspace(size_t bytes) {
    if (bytes <= workspace.bytes) return;
    if (workspace.ptr) detail::release(workspace);
    workspace = detail::allocate(bytes);
  }

  // TL_FLAT_ALLREDUCE=1: the packed all-reduce (one NCCL call over one
  // flat buffer) instead of one NCCL group of per-tensor all-reduces.
  static bool flat_allreduce() {
    static const bool on = [] {
      const char *e = std::getenv("TL_FLAT_ALLREDUCE");
      return e && std::strcmp(e, "1") == 0;
    }();
    return on;
  }

  void ensure_flat(size_t bytes) {
    if (bytes <= flat_dev.bytes) return;
    if (flat_dev.ptr) detail::release(flat_dev);
    flat_dev = detail::allocate(bytes);
  }

  // The all-reduce's slot table (gradient, count, chunk0 per tensor);
  // returns the chunk count of the packed layout.
  uint32_t stage_grad_slots(const Op &op, size_t base) {
    tl_param_slot *h = static_cast<tl_param_slot *>(slot_host) + base;
    uint32_t chunk = 0;
    for (size_t i = 0; i < op.multi.size(); ++i) {
      h[i] = tl_param_slot{};
      h[i].grad = op.multi[i].grad.f();
      h[i].count = op.multi[i].grad.numel();
      h[i].chunk0 = chunk;
      chunk += static_cast<uint32_t>((h[i].count + TL_OPT_CHUNK - 1) / TL_OPT_CHUNK);
    }
    return chunk;
  }

  void ensure_slots(size_t count) {
    if (count <= slot_capacity) return;
    if (slot_dev.ptr) detail::release(slot_dev);
    if (slot_host) tl_host_free(slot_host);
    slot_host = nullptr;
    const size_t bytes = count * sizeof(tl_param_slot);
    slot_dev = detail::allocate(bytes);
    check(tl_host_alloc(&slot_host, bytes), "optimiser slot staging");
    slot_capacity = count;
  }

  // Fills the pinned slot table of a fused optimiser op; returns chunk count.
  uint32_t stage_slots(const Op &op, size_t base) {
    tl_param_slot *h = static_cast<tl_param_slot *>(slot_host) + base;
    uint32_t chunk = 0;
    for (size_t i = 0; i < op.multi.size(); ++i) {
      const auto &s = op.multi[i];
      h[i].param = s.param.f();
      h[i].out = s.out.f();
      h[i].grad = s.grad.f();
      h[i].m1 = s.m1.f();
      h[i].m2 = s.m2.f();
      h[i].count = s.param.numel();
      h[i].chunk0 = chunk;
      h[i].step = s.step;
      chunk += static_cast<uint32_t>((h[i].count + TL_OPT_CHUNK - 1) / TL_OPT_CHUNK);
    }
    return chunk;
  }

  void execute(const Op &op, void *s, size_t slot_base) {
    void *ws = workspace.ptr;
    const size_t wsb = workspace.bytes;
    const TRef *t = op.t.data();
    switch (op.kind) {
      case Kind::Binary:
        check(tl_binary(op.code, t[0].f(), t[0].shape, t[0].rank, t[1].f(), t[1].shape, t[1].rank,
                        t[2].f(), t[2].shape, t[2].rank, s),
              "binary op");
        break;
      case Kind::Scalar:
        check(tl_scalar(op.code, t[0].f(), op.f0, t[1].f(), t[1].numel(), s), "scalar op");
        break;
      case Kind::Unary:
        check(tl_unary(op.code, t[0].f(), t[1].f(), t[1].numel(), s), "unary op");
        break;
      case Kind::Copy:
        check(tl_copy(t[0].f(), t[1].f(), t[1].numel(), s), "copy");
        break;
      case Kind::Reduce:
        if (!op.group_refs.empty()) {  // same-shape reductions grouped by the optimiser
          const float *xs[TL_REDUCE_MAX_GROUPS] = {t[0].f()};
          float *outs[TL_REDUCE_MAX_GROUPS] = {t[1].f()};
          uint32_t n = 1;
          for (size_t k = 0; k + 1 < op.group_refs.size() && n < TL_REDUCE_MAX_GROUPS; k += 2, ++n) {
            xs[n] = op.group_refs[k].f();
            outs[n] = op.group_refs[k + 1].f();
          }
          check(tl_reduce_group(op.code, n, xs, t[0].shape, t[0].rank, outs, t[1].shape,
                                t[1].rank, ws, wsb, s),
                "reduce group");
          break;
        }
        check(tl_reduce(op.code, t[0].f(), t[0].shape, t[0].rank, t[1].f(), t[1].shape, t[1].rank,
                        ws, wsb, s),
              "reduce");
        break;
      case Kind::Argmax:
        check(tl_argmax(t[0].f(), t[0].numel(), t[1].u(), ws, wsb, s), "argmax");
        break;
      case Kind::Transpose:
        check(tl_transpose(t[0].f(), t[0].shape, t[0].rank, op.i0, op.i1, t[1].f(), s),
              "transpose");
        break;
      case Kind::Softmax:
        if (t[2].p || t[3].p)
          check(tl_softmax_scaled_masked_rows(
                    t[0].f(), t[2].p ? t[2].f() : nullptr, t[3].p ? t[3].f() : nullptr,
                    t[3].p ? static_cast<uint32_t>(t[3].numel() / t[0].last()) : 0u, t[1].f(),
                    static_cast<uint32_t>(t[0].numel() / t[0].last()), t[0].last(), s),
                "softmax");
        else
          check(tl_softmax_rows(t[0].f(), t[1].f(),
                                static_cast<uint32_t>(t[0].numel() / t[0].last()), t[0].last(), s),
                "softmax");
        break;
      case Kind::Rms:
        check(tl_rms_rows(t[0].f(), t[1].f(), static_cast<uint32_t>(t[0].numel() / t[0].last()),
                          t[0].last(), s),
              "RMS");
        break;
      case Kind::RmsNorm:
        check(tl_rmsnorm_rows(t[0].f(), t[1].f(), nullptr,
                              static_cast<uint32_t>(t[0].numel() / t[0].last()), t[0].last(), s),
              "RMSNorm");
        break;
      case Kind::Xent:
        check(tl_xent_rows(t[0].f(), t[1].u(), t[2].f(), static_cast<uint32_t>(t[1].numel()),
                           t[0].last(), s),
              "cross_entropy");
        break;
      case Kind::XentBwd:
        check(tl_xent_backward_rows(t[0].f(), t[1].u(), t[3].p ? t[3].f() : nullptr, t[2].f(),
                                    static_cast<uint32_t>(t[1].numel()), t[0].last(), s),
              "cross_entropy_derivative");
        break;
      case Kind::Gather:
        check(tl_embedding_gather(t[0].f(), t[0].shape[0], t[0].shape[1], t[1].u(),
                                  static_cast<uint32_t>(t[1].numel()), t[2].f(), s),
              "embedding_lookup");
        break;
      case Kind::Scatter:
        check(tl_embedding_scatter_add(t[0].f(), t[1].u(), static_cast<uint32_t>(t[1].numel()),
                                       t[3].shape[1], t[2].p ? t[2].f() : nullptr, t[3].f(),
                                       t[3].shape[0], ws, wsb, s),
              "scatter");
        break;
      case Kind::SqNorm:
        check(tl_grad_sqnorm_accumulate(t[0].f(), t[0].numel(), t[1].f(), ws, wsb, s),
              "accumulate_gradient_squared_norm");
        break;
      case Kind::Clip:
        check(tl_clip_gradient(t[0].f(), t[1].f(), op.f0, t[2].f(), t[2].numel(), s),
              "clip_gradient");
        break;
      case Kind::AdamW:
        check(tl_adamw(t[0].f(), t[1].f(), t[2].f(), t[3].f(), t[4].f(), t[5].f(), t[6].f(),
                       t[7].f(), t[8].f(), op.f0, op.u0, t[0].numel(), s),
              "adamW");
        break;
      case Kind::Gemm: {
        tl_gemm_desc d = op.gemm;
        d.workspace = ws;
        d.workspace_bytes = wsb;
        check(tl_gemm(&d, s), "mult");
        break;
      }
      case Kind::HostWrite:
        check(tl_memcpy_h2d(static_cast<char *>(t[0].p) + op.n, op.host.data(), op.host.size(), s),
              "Storage::write");
        break;
      case Kind::Fill:
        check(tl_fill_u32(t[0].p, op.u0, op.n, s), "Storage::fill");
        break;
      case Kind::DevCopy:
        check(tl_memcpy_d2d(t[0].p, t[1].p, op.n, s), "Storage::clone");
        break;
      case Kind::Release:
        break;
      case Kind::GeluBwd:
        check(tl_gelu_backward(t[0].f(), t[1].f(), t[2].f(), t[2].numel(), s), "GELU backward");
        break;
      case Kind::SoftmaxBwd:
        check(tl_softmax_backward_rows(t[0].f(), t[1].f(), t[3].p ? t[3].f() : nullptr, t[2].f(),
                                       static_cast<uint32_t>(t[2].numel() / t[2].last()),
                                       t[2].last(), s),
              "softmax backward");
        break;
      case Kind::RmsNormBwd:
        check(tl_rmsnorm_backward_rows(t[0].f(), t[1].f(), t[2].f(), t[4].p ? t[4].f() : nullptr,
                                       t[3].f(),
                                       static_cast<uint32_t>(t[3].numel() / t[3].last()),
                                       t[3].last(), s),
              "RMSNorm backward");
        break;
      case Kind::MultiAdamW: {
        const uint32_t chunks = stage_slots(op, slot_base);
        tl_param_slot *dev = static_cast<tl_param_slot *>(slot_dev.ptr) + slot_base;
        check(tl_memcpy_h2d(dev, static_cast<tl_param_slot *>(slot_host) + slot_base,
                            op.multi.size() * sizeof(tl_param_slot), s),
              "optimiser slots");
        check(tl_multi_clip_adamw(dev, static_cast<uint32_t>(op.multi.size()), chunks,
                                  t[0].p ? t[0].f() : nullptr, op.f0, t[5].f(), t[6].f(),
                                  t[7].f(), t[8].f(), op.f1, ws, wsb, s),
              "fused clip + AdamW");
        break;
      }
      case Kind::AllReduce: {
        if (!flat_allreduce()) {
          internal::all_reduce_gradients(op, comm, s);
          break;
        }
        // pack every gradient into one buffer, one NCCL sum, unpack
        const uint32_t chunks = stage_grad_slots(op, slot_base);
        tl_param_slot *dev = static_cast<tl_param_slot *>(slot_dev.ptr) + slot_base;
        check(tl_memcpy_h2d(dev, static_cast<tl_param_slot *>(slot_host) + slot_base,
                            op.multi.size() * sizeof(tl_param_slot), s),
              "all-reduce slots");
        const uint32_t n = static_cast<uint32_t>(op.multi.size());
        float *flat = static_cast<float *>(flat_dev.ptr);
        check(tl_multi_grad_flat(dev, n, chunks, flat, 0, s), "gradient pack");
        internal::all_reduce_flat(flat, static_cast<size_t>(chunks) * TL_OPT_CHUNK, comm, s);
        check(tl_multi_grad_flat(dev, n, chunks, flat, 1, s), "gradient unpack");
        break;
      }
      case Kind::Attention: {
        tl_attn_desc d = op.attn;
        d.workspace = ws;
        d.workspace_bytes = wsb;
        if (d.pass == TL_ATTN_FORWARD && d.mask_flag && (op.u0 & 1))
          check(tl_attention_mask_check(d.mask, d.T, const_cast<uint32_t *>(d.mask_flag), s),
                "attention mask check");
        check(tl_attention_fused(&d, s), "attention");
        break;
      }
      case Kind::FlashFwd:
        if (op.code & 1)
          check(tl_attention_mask_check(op.flash.mask, op.flash.T,
                                        const_cast<uint32_t *>(op.flash.mask_flag), s),
                "attention mask check");
        check(tl_flash_attention_fwd(&op.flash, s), "flash attention");
        break;
      case Kind::FlashBwd: {
        tl_flash_desc d = op.flash;
        d.delta = static_cast<float *>(ws);
        check(tl_flash_attention_bwd(&d, s), "flash attention backward");
        break;
      }
      case Kind::FlashProbs:
        check(tl_flash_attention_probs(&op.flash, t[4].f(), s), "flash attention P");
        break;
    }
  }

  // Signature of a program for graph reuse: everything a launch depends on
  // except the values graphs re-read at replay (optimiser slot tables).
  static std::string signature(const std::vector<Op> &p) {
    std::string sig;
    sig.reserve(p.size() * 96);
    auto put = [&](const void *d, size_t n) { sig.append(static_cast<const char *>(d), n); };
    for (const Op &op : p) {
      if (op.dead || op.kind == Kind::Release) continue;
      put(&op.kind, sizeof(op.kind));
      put(&op.code, sizeof(op.code));
      for (const TRef &r : op.t) {
        if (!r.p) continue;
        put(&r.p, sizeof(r.p));
        put(&r.rank, 1);
        put(r.shape, r.rank * sizeof(uint32_t));
      }
      put(&op.f0, sizeof(float));
      put(&op.f1, sizeof(float));
      put(&op.i0, sizeof(int32_t));
      put(&op.i1, sizeof(int32_t));
      put(&op.n, sizeof(op.n));
      if (op.kind == Kind::AdamW) put(&op.u0, sizeof(op.u0));
      if (op.kind == Kind::Fill) put(&op.u0, sizeof(op.u0));
      if (op.kind == Kind::Gemm) put(&op.gemm, sizeof(op.gemm));
      if (op.kind == Kind::Attention) put(&op.attn, sizeof(op.attn));
      if (op.kind == Kind::FlashFwd || op.kind == Kind::FlashBwd || op.kind == Kind::FlashProbs)
        put(&op.flash, sizeof(op.flash));
      if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) {
        for (const auto &s : op.multi) {
          put(&s.param.p, sizeof(void *));
          put(&s.grad.p, sizeof(void *));
          put(&s.out.p, sizeof(void *));
          put(&s.m1.p, sizeof(void *));
          put(&s.m2.p, sizeof(void *));
        }
      }
    }
    return sig;
  }

  static bool capturable(const std::vector<Op> &p) {
    for (const Op &op : p)
      if (!op.dead && (op.kind == Kind::HostWrite || op.kind == Kind::AllReduce)) return false;
    return true;
  }

  void run_ops(void *s) {
    size_t slot_base = 0;
    for (const Op &op : prog) {
      if (op.dead) continue;
      execute(op, s, slot_base);
      if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce)
        slot_base += op.multi.size();
    }
  }

  // Per-op device time: one event between consecutive ops, all enqueued
  // before the first is read, so the GPU runs the program back to back
  // (an op's time can include host launch latency only when the GPU ran
  // dry waiting for it).
  static std::string profile_key(const Op &op) {
    std::string key = internal::kind_name(op.kind);
    if (op.kind == Kind::Gemm) {
      key += " " + std::to_string(op.gemm.m) + "x" + std::to_string(op.gemm.n) + "x" +
             std::to_string(op.gemm.k);
      uint64_t batch = 1;
      for (uint32_t i = 0; i < op.gemm.batch_rank; ++i) batch *= op.gemm.batch_shape[i];
      if (batch > 1) key += " b" + std::to_string(batch);
      key += op.gemm.trans_a ? " T" : " N";
      key += op.gemm.trans_b ? "T" : "N";
      if (op.gemm.groups > 1) key += " g" + std::to_string(op.gemm.groups);
      if (op.gemm.c_heads) key += " heads";
    } else if (op.kind == Kind::Attention) {
      key += "#" + std::to_string(op.code) + " " + std::to_string(op.attn.B) + "x" +
             std::to_string(op.attn.H) + "x" + std::to_string(op.attn.T) + "x" +
             std::to_string(op.attn.D);
    } else if (op.kind == Kind::FlashFwd || op.kind == Kind::FlashBwd ||
               op.kind == Kind::FlashProbs) {
      key += " " + std::to_string(op.flash.B) + "x" + std::to_string(op.flash.H) + "x" +
             std::to_string(op.flash.T) + "x" + std::to_string(op.flash.D);
    } else if (op.kind != Kind::MultiAdamW && op.kind != Kind::AllReduce) {
      // element-wise and row ops: code and the shapes that set the traffic
      if (op.kind == Kind::Binary || op.kind == Kind::Unary || op.kind == Kind::Scalar ||
          op.kind == Kind::Reduce)
        key += "#" + std::to_string(op.code);
      if (op.kind == Kind::Reduce && !op.group_refs.empty())
        key += " g" + std::to_string(1 + op.group_refs.size() / 2);
      for (int i = 0; i < 3; ++i) {
        const TRef &r = op.t[i];
        if (!r.p || r.rank == 0) continue;
        key += " [";
        for (int d = 0; d < r.rank; ++d) key += (d ? "," : "") + std::to_string(r.shape[d]);
        key += "]";
      }
    }
    return key;
  }

  // Algorithmic bytes of a memory-bound op: every operand it reads read
  // once and every output written once (an in-place operand counts twice);
  // 0 for the tensor-core ops and data movement.
  static double op_bytes(const Op &op) {
    switch (op.kind) {
      case Kind::Gemm: case Kind::Attention: case Kind::FlashFwd: case Kind::FlashBwd:
      case Kind::FlashProbs: case Kind::AllReduce: case Kind::HostWrite: case Kind::Release:
        return 0.0;
      case Kind::MultiAdamW: {
        double n = 0.0;
        for (const internal::MultiSlot &m : op.multi) n += static_cast<double>(m.param.numel());
        // param, grad, m1, m2 read; out, m1, m2 written; + the norm's read
        return n * 4.0 * (7.0 + (op.t[0].p ? 1.0 : 0.0));
      }
      default: {
        double b = 0.0;
        for (const TRef &r : op.t)
          if (r.p) b += static_cast<double>(r.numel()) * 4.0;
        for (const TRef &r : op.group_refs)  // grouped reductions
          if (r.p) b += static_cast<double>(r.numel()) * 4.0;
        return b;
      }
    }
  }

  void run_profiled(void *s) {
    std::vector<const Op *> ops;
    for (const Op &op : prog)
      if (!op.dead && op.kind != Kind::Release) ops.push_back(&op);
    std::vector<void *> ev(ops.size() + 1, nullptr);
    for (void *&e : ev) check(tl_event_create(&e), "profile event");
    size_t slot_base = 0;
    for (size_t i = 0; i < ops.size(); ++i) {
      check(tl_event_record(ev[i], s), "profile event");
      execute(*ops[i], s, slot_base);
      if (ops[i]->kind == Kind::MultiAdamW || ops[i]->kind == Kind::AllReduce)
        slot_base += ops[i]->multi.size();
    }
    check(tl_event_record(ev.back(), s), "profile event");
    for (size_t i = 0; i < ops.size(); ++i) {
      float ms = 0.0f;
      check(tl_event_elapsed_ms(&ms, ev[i], ev[i + 1]), "profile event");
      Prof &p = profile[profile_key(*ops[i])];
      ++p.calls;
      p.ms += ms;
      p.bytes += op_bytes(*ops[i]);
    }
    for (void *e : ev) tl_event_destroy(e);
  }

  void run_program() {
    void *s = cuda::stream();
    size_t ws = 0, slots = 0, flat_chunks = 0;
    uint64_t live = 0;
    for (const Op &op : prog) {
      if (op.dead) continue;
      ws = std::max(ws, op.kind == Kind::Gemm ? tl_gemm_workspace_size(&op.gemm) : op.workspace);
      if (op.kind == Kind::MultiAdamW || op.kind == Kind::AllReduce) slots += op.multi.size();
      if (op.kind == Kind::AllReduce) {
        size_t c = 0;
        for (const auto &m : op.multi) c += (m.grad.numel() + TL_OPT_CHUNK - 1) / TL_OPT_CHUNK;
        flat_chunks = std::max(flat_chunks, c);
      }
      if (op.kind != Kind::Release) ++live;
    }
    ensure_workspace(ws);
    if (slots) ensure_slots(slots);
    if (flat_chunks && flat_allreduce()) ensure_flat(flat_chunks * TL_OPT_CHUNK * sizeof(float));
    stats.ops_launched += live;
    const uint64_t k0 = tl_kernel_launches();
    if (profiling) {
      run_profiled(s);
      stats.kernel_launches += tl_kernel_launches() - k0;
      return;
    }
    if (!graphs || !capturable(prog)) {
      run_ops(s);
      stats.kernel_launches += tl_kernel_launches() - k0;
      return;
    }
    std::string sig = planned_sig ? *planned_sig : signature(prog);
    auto it = graph_cache.find(sig);
    if (it != graph_cache.end()) {
      // slot tables are re-read from pinned memory by the graph's copies
      size_t base = 0;
      for (const Op &op : prog)
        if (!op.dead && op.kind == Kind::MultiAdamW) {
          stage_slots(op, base);
          base += op.multi.size();
        }
      check(tl_graph_launch(it->second.exec, s), "graph replay");
      it->second.last_use = ++use_clock;
      ++stats.graph_replays;
      stats.kernel_launches += it->second.kernels;
      return;
    }
    if (seen_once.find(sig) == seen_once.end()) {
      // first sighting: run eagerly, capture if the same program comes back
      if (seen_once.size() >= 64) seen_once.clear();
      seen_once.emplace(std::move(sig), ++use_clock);
      run_ops(s);
      stats.kernel_launches += tl_kernel_launches() - k0;
      return;
    }
    seen_once.erase(sig);
    check(tl_graph_capture_begin(s), "graph capture");
    try {
      run_ops(s);
    } catch (...) {
      void *junk = nullptr;
      tl_graph_capture_end(s, &junk);
      tl_graph_destroy(junk);
      throw;
    }
    void *exec = nullptr;
    check(tl_graph_capture_end(s, &exec), "graph capture");
    const uint64_t kernels = tl_kernel_launches() - k0;
    if (graph_cache.size() >= 8) {
      auto victim = std::min_element(graph_cache.begin(), graph_cache.end(),
                                     [](const auto &a, const auto &b) {
                                       return a.second.last_use < b.second.last_use;
                                     });
      tl_graph_destroy(victim->second.exec);
      graph_cache.erase(victim);
    }
    graph_cache[std::move(sig)] = Cached{exec, kernels, ++use_clock};
    ++stats.graph_captures;
    check(tl_graph_launch(exec, s), "graph launch");
    stats.kernel_launches += kernels;
  }

  void write_profile() {
    std::ofstream out(profile_path);
    out << "{\n  \"ops\": [\n";
    bool first = true;
    for (const auto &kv : profile) {
      out << (first ? "" : ",\n") << "    {\"op\": \"" << kv.first << "\", \"calls\": "
          << kv.second.calls << ", \"ms\": " << kv.second.ms
          << ", \"bytes\": " << static_cast<uint64_t>(kv.second.bytes) << "}";
      first = false;
    }
    out << "\n  ]\n}\n";
  }
};

// ---------------------------------------------------------------- lifecycle
Runtime::Runtime() : impl_(std::make_unique<Impl>()) {
  internal::ensure_init();
  internal::add_host_access_hook(impl_.get());
}

Runtime::~Runtime() {
  cleanup();
  internal::remove_host_access_hook(impl_.get());
}

// src/my_metal/runtime.cpp:290-297
void Runtime::start() {
  if (impl_->state != Impl::State::Idle)
    throw std::logic_error("CUDA runtime execution already started");
  impl_->prog.clear();
  impl_->window_id = internal::next_window_id();
  impl_->state = Impl::State::Recording;
  impl_->record_t0 = std::chrono::steady_clock::now();
  internal::set_active_recorder(impl_.get());
}

// src/my_metal/runtime.cpp:299-309
void Runtime::submit() {
  if (impl_->state != Impl::State::Recording)
    throw std::logic_error("CUDA runtime execution has not started");
  if (internal::active_recorder() == impl_.get()) internal::set_active_recorder(nullptr);
  cuda::detail::device_changed();  // this window's launches may write anything
  const auto t_submit = std::chrono::steady_clock::now();
  impl_->stats.host_record_ns += static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::nanoseconds>(t_submit - impl_->record_t0).count());
  bool dump = false;
  if (!impl_->dump_path.empty() && impl_->dumped.size() < 64) {
    std::string key = Impl::signature(impl_->prog);
    key += impl_->optimizer_windows >= 2 ? 'L' : '-';  // window liveness known
    dump = impl_->dumped.insert(std::move(key)).second;
    if (dump) impl_->dump("recorded", true);
  }
  const uint64_t recorded_ops = impl_->prog.size();
  impl_->planned_sig = nullptr;
  if (impl_->fusion) impl_->optimise_program();
  else if (impl_->comm) internal::add_gradient_allreduce(impl_->prog);
  if (dump) impl_->dump("optimised", true);
  const auto t_optimised = std::chrono::steady_clock::now();
  impl_->state = Impl::State::Submitted;
  ++impl_->stats.windows;
  try {
    impl_->run_program();
  } catch (...) {
    impl_->prog.clear();
    throw;
  }
  if (impl_->flash) {
    for (const Op &op : impl_->prog) {
      if (op.dead) continue;
      impl_->stats.flash_forward += op.kind == Kind::FlashFwd;
      impl_->stats.flash_backward += op.kind == Kind::FlashBwd;
      impl_->stats.flash_rebuilt += op.kind == Kind::FlashProbs;
    }
    internal::update_flash_records(impl_->prog, impl_->flash_records);
  }
  impl_->prog.clear();
  if (!impl_->trace_path.empty()) {
    const auto now = std::chrono::steady_clock::now();
    auto ns = [](auto d) {
      return static_cast<uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(d).count());
    };
    impl_->trace.push_back({recorded_ops, ns(t_submit - impl_->record_t0),
                            ns(t_optimised - t_submit), ns(now - t_optimised)});
  }
  impl_->stats.host_submit_ns += static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() -
                                                           t_submit)
          .count());
}

// src/my_metal/runtime.cpp:310-317
void Runtime::wait() {
  if (impl_->state != Impl::State::Submitted)
    throw std::logic_error("CUDA runtime execution has not been submitted");
  impl_->state = Impl::State::Idle;
  uint32_t flags = 0;
  if (impl_->deferred_wait) flags = impl_->deferred_status();
  else check(tl_device_status(&flags, cuda::stream()), "CUDA runtime wait");
  if (flags & TL_FLAG_INDEX_RANGE)
    throw std::out_of_range("embedding index out of range of the embedding table");
  if (flags & TL_FLAG_TIMEOUT)
    throw std::runtime_error("a CUDA kernel gave up waiting on the device (timeout)");
}

// src/my_metal/runtime.cpp:170-177
void Runtime::abort() noexcept {
  if (internal::active_recorder() == impl_.get()) internal::set_active_recorder(nullptr);
  impl_->prog.clear();
  impl_->state = Impl::State::Idle;
}

// src/my_metal/runtime.cpp:179-230
void Runtime::cleanup() noexcept {
  if (!impl_) return;
  if (impl_->state == Impl::State::Recording) abort();
  if (impl_->state == Impl::State::Submitted) {
    tl_stream_sync(cuda::initialised() ? cuda::stream() : nullptr);
    impl_->state = Impl::State::Idle;
  }
  if (cuda::initialised()) {
    tl_stream_sync(cuda::stream());
    impl_->release_resources();
  }
}

// src/my_metal/runtime.cpp:42-63
void Runtime::start_profile(std::string_view output_path) {
  impl_->profiling = true;
  impl_->profile_path = std::string(output_path);
  impl_->profile.clear();
}

void Runtime::end_profile() {
  if (!impl_->profiling) return;
  impl_->profiling = false;
  impl_->write_profile();
}

void Runtime::set_fusion(bool enabled) { impl_->fusion = enabled; }
void Runtime::set_flash_attention(int mode) {
  if (mode < 0 || mode > 2) throw std::invalid_argument("flash attention mode is 0, 1 or 2");
  impl_->flash = mode;
}
void Runtime::set_deferred_wait(bool enabled) { impl_->deferred_wait = enabled; }
void Runtime::set_graphs(bool enabled) { impl_->graphs = enabled; }
void Runtime::set_gemm_precision(int precision) {
  if (precision != TL_GEMM_TF32 && precision != TL_GEMM_FP32 && precision != TL_GEMM_3XTF32)
    throw std::invalid_argument("unsupported GEMM precision");
  impl_->gemm_precision = precision;
}
void Runtime::set_communicator(void *nccl_comm) { impl_->comm = nccl_comm; }
const RuntimeStats &Runtime::stats() const { return impl_->stats; }

// ---------------------------------------------------------------- elementwise
namespace {
void binary(Runtime::Impl &im, int code, const Mat &a, const Mat &b, Mat &out) {
  check_broadcast(a.shape(), out.shape());
  check_broadcast(b.shape(), out.shape());
  Op &op = im.record(Kind::Binary);
  op.code = code;
  op.t[0] = ref(a);
  op.t[1] = ref(b);
  op.t[2] = ref(out);
}

// src/my_metal/runtime.cpp:116-136
void scalar(Runtime::Impl &im, int code, const Mat &a, float s, Mat &out) {
  if (a.shape() != out.shape())
    throw std::invalid_argument("scalar operation input and output shapes must match");
  Op &op = im.record(Kind::Scalar);
  op.code = code;
  op.t[0] = ref(a);
  op.t[1] = ref(out);
  op.f0 = s;
}

// src/my_metal/runtime.cpp:97-114 (dispatched over the output's elements)
void unary(Runtime::Impl &im, int code, const Mat &a, Mat &out) {
  if (a.numel() != out.numel())
    throw std::invalid_argument("unary operation input and output sizes must match");
  Op &op = im.record(Kind::Unary);
  op.code = code;
  op.t[0] = ref(a);
  op.t[1] = ref(out);
}
}  // namespace

// src/my_metal/runtime.cpp:321-353
void Runtime::add(const Mat &a, const Mat &b, Mat &o) { binary(*impl_, TL_ADD, a, b, o); }
void Runtime::add(const Mat &a, kernel_type s, Mat &o) { scalar(*impl_, TL_SCALAR_ADD, a, s, o); }
void Runtime::sub(const Mat &a, const Mat &b, Mat &o) { binary(*impl_, TL_SUB, a, b, o); }
void Runtime::hadamard(const Mat &a, const Mat &b, Mat &o) { binary(*impl_, TL_MUL, a, b, o); }
void Runtime::divide(const Mat &a, const Mat &b, Mat &o) { binary(*impl_, TL_DIV, a, b, o); }
void Runtime::divide(const Mat &a, kernel_type s, Mat &o) {
  scalar(*impl_, TL_SCALAR_DIV, a, s, o);
}
// src/my_metal/runtime.cpp:355-373
void Runtime::sigmoid(const Mat &a, Mat &o) { unary(*impl_, TL_SIGMOID, a, o); }
void Runtime::sqrt(const Mat &a, Mat &o) { unary(*impl_, TL_SQRT, a, o); }
void Runtime::pow(const Mat &a, kernel_type e, Mat &o) { scalar(*impl_, TL_SCALAR_POW, a, e, o); }
void Runtime::exp(const Mat &a, Mat &o) { unary(*impl_, TL_EXP, a, o); }
// src/my_metal/runtime.cpp:1073-1081
void Runtime::GELU(const Mat &a, Mat &o) { unary(*impl_, TL_GELU, a, o); }
void Runtime::GELU_derivative(const Mat &a, Mat &o) { unary(*impl_, TL_GELU_DERIVATIVE, a, o); }

// src/my_metal/runtime.cpp:1170-1186
void Runtime::copy(const Mat &a, Mat &output) {
  if (a.shape() != output.shape())
    throw std::invalid_argument("copy destination has incorrect shape");
  Op &op = impl_->record(Kind::Copy);
  op.t[0] = ref(a);
  op.t[1] = ref(output);
}

// src/my_metal/runtime.cpp:843-848
void Runtime::sqe(const Mat &pred, const Mat &target, Mat &output) {
  sub(pred, target, output);
  hadamard(output, output, output);
}

// ----------------------------------------------------------------------- GEMM
// src/my_metal/runtime.cpp:375-505: C = A*B over the last two dims with
// broadcast batch dims.
void Runtime::mult(const Mat &a, const Mat &b, Mat &output) {
  const auto expected = rtensor::infer_mult(a.shape(), b.shape());  // same throws as Metal
  if (output.shape() != expected)
    throw std::invalid_argument("matmul destination has incorrect shape");
  Op &op = impl_->record(Kind::Gemm);
  op.t[0] = ref(a);
  op.t[1] = ref(b);
  op.t[2] = ref(output);
  tl_gemm_desc &g = op.gemm;
  const auto &as = a.shape(), &bs = b.shape(), &cs = output.shape();
  g.a = static_cast<const float *>(op.t[0].p);
  g.b = static_cast<const float *>(op.t[1].p);
  g.c = op.t[2].f();
  g.m = as[as.size() - 2];
  g.k = as[as.size() - 1];
  g.n = bs[bs.size() - 1];
  g.precision = impl_->gemm_precision;
  const size_t batch_rank = cs.size() - 2;
  // merge batch dims into at most TL_GEMM_MAX_BATCH_RANK (they are dense)
  std::vector<uint32_t> bshape;
  std::vector<uint64_t> sa, sb, sc;
  const uint64_t amat = uint64_t(g.m) * g.k, bmat = uint64_t(g.k) * g.n, cmat = uint64_t(g.m) * g.n;
  auto dense_strides = [&](const std::vector<uint32_t> &shape, size_t rank, uint64_t mat) {
    std::vector<uint64_t> st(batch_rank, 0);
    const size_t r = shape.size() - 2;
    uint64_t acc = mat;
    for (size_t i = r; i-- > 0;) {
      const size_t oi = batch_rank - r + i;
      st[oi] = shape[i] == 1 ? 0 : acc;
      acc *= shape[i];
    }
    (void)rank;
    return st;
  };
  const auto full_a = dense_strides(as, as.size(), amat);
  const auto full_b = dense_strides(bs, bs.size(), bmat);
  const auto full_c = dense_strides(cs, cs.size(), cmat);
  for (size_t i = 0; i < batch_rank; ++i) {
    if (cs[i] == 1) continue;
    if (!bshape.empty() && sa.back() == full_a[i] * cs[i] && sb.back() == full_b[i] * cs[i] &&
        sc.back() == full_c[i] * cs[i]) {
      bshape.back() *= cs[i];
      sa.back() = full_a[i];
      sb.back() = full_b[i];
      sc.back() = full_c[i];
      continue;
    }
    bshape.push_back(cs[i]);
    sa.push_back(full_a[i]);
    sb.push_back(full_b[i]);
    sc.push_back(full_c[i]);
  }
  if (bshape.size() > TL_GEMM_MAX_BATCH_RANK)
    throw std::invalid_argument("matmul batch rank exceeds the CUDA runtime limit");
  // A batch of row-blocks against one shared B (activations x weights,
  // e.g. [64,192,384] x [384,384]) is a single product with M * batch rows.
  if (bshape.size() == 1 && sb[0] == 0 && sa[0] == amat && sc[0] == cmat) {
    g.m *= bshape[0];
    bshape.clear();
    op.i1 = 1;  // flattened: A's rows run across the batch
  }
  g.batch_rank = static_cast<uint32_t>(bshape.size());
  for (size_t i = 0; i < bshape.size(); ++i) {
    g.batch_shape[i] = bshape[i];
    g.a_batch_stride[i] = sa[i];
    g.b_batch_stride[i] = sb[i];
    g.c_batch_stride[i] = sc[i];
  }
}

// --------------------------------------------------------------- reductions
// src/my_metal/runtime.cpp:506-518
void Runtime::sum(const Mat &input, Mat &output) {
  if (output.numel() < 1) throw std::invalid_argument("sum destination must hold a value");
  Op &op = impl_->record(Kind::Reduce);
  op.code = TL_REDUCE_SUM;
  op.t[0] = ref(input);
  op.t[1] = ref(output);
  op.t[1].rank = 1;
  op.t[1].shape[0] = 1;
  op.workspace = tl_reduce_workspace_size(op.t[0].shape, op.t[0].rank, op.t[1].shape, 1);
}

// src/my_metal/runtime.cpp:520-527
void Runtime::sum(const Mat &input, size_t axis, Mat &output) {
  if (axis >= input.shape().size()) throw std::out_of_range("sum axis out of range");
  sum_to_shape(input, output.shape(), output);
}

// src/my_metal/runtime.cpp:661-739
void Runtime::sum_to_shape(const Mat &a, std::span<const uint32_t> output_shape, Mat &output) {
  const auto &a_shape = a.shape();
  if (output_shape.size() > a_shape.size())
    throw std::invalid_argument("cannot reduce to a shape with a higher rank");
  if (output.shape().size() != output_shape.size() ||
      !std::equal(output.shape().begin(), output.shape().end(), output_shape.begin()))
    throw std::invalid_argument("sum_to_shape destination has incorrect shape");
  const size_t off = a_shape.size() - output_shape.size();
  bool reduced = false;
  for (size_t i = 0; i < a_shape.size(); ++i) {
    const uint32_t o = i < off ? 1u : output_shape[i - off];
    if (a_shape[i] != o) {
      if (o != 1) throw std::invalid_argument("invalid reduce_to_shape");
      reduced = true;
    }
  }
  if (!reduced) {  // same element order: a copy (Metal adds 0 through a view)
    Op &op = impl_->record(Kind::Copy);
    op.t[0] = ref(a);
    op.t[1] = ref(output);
    return;
  }
  Op &op = impl_->record(Kind::Reduce);
  op.code = TL_REDUCE_SUM;
  op.t[0] = ref(a);
  op.t[1] = ref(output);
  op.workspace = tl_reduce_workspace_size(op.t[0].shape, op.t[0].rank, op.t[1].shape,
                                          op.t[1].rank);
}

// src/my_metal/runtime.cpp:595-659
void Runtime::reduce_to_shape(const Mat &a, std::span<const uint32_t> output_shape, Mat &output,
                              ReduceKind kind) {
  if (output_shape.size() != a.shape().size())
    throw std::invalid_argument("cannot reduce to shape if ranks differ");
  size_t shrink = 0;
  for (size_t i = 0; i < output_shape.size(); ++i) {
    if (a.shape()[i] != output_shape[i]) {
      if (output_shape[i] != 1) throw std::invalid_argument("invalid reduce_to_shape");
      if (++shrink > 1)
        throw std::invalid_argument(
            "reduce_to_shape currently supports only one shrinking dimension");
    }
  }
  if (shrink == 0) {
    output = a;
    return;
  }
  Op &op = impl_->record(Kind::Reduce);
  op.code = kind == ReduceKind::Sum ? TL_REDUCE_SUM : TL_REDUCE_MAX;
  op.t[0] = ref(a);
  op.t[1] = ref(output);
  op.workspace = tl_reduce_workspace_size(op.t[0].shape, op.t[0].rank, op.t[1].shape,
                                          op.t[1].rank);
}

// src/my_metal/runtime.cpp:741-745
void Runtime::max_to_shape(const Mat &a, std::span<const uint32_t> output_shape, Mat &output) {
  reduce_to_shape(a, output_shape, output, ReduceKind::Max);
}

// src/my_metal/runtime.cpp:850-918
void Runtime::argmax(const Mat &a, IndexMat &output) {
  if (a.numel() == 0) throw std::invalid_argument("argmax requires a non-empty tensor");
  if (output.numel() < 1) throw std::invalid_argument("argmax destination must hold an index");
  Op &op = impl_->record(Kind::Argmax);
  op.t[0] = ref(a);
  op.t[1] = ref(output);
  op.workspace = tl_argmax_workspace_size(a.numel());
}

// ---------------------------------------------------------------- layout ops
// src/my_metal/runtime.cpp:529-569
void Runtime::transpose(const Mat &a, Mat &output, int32_t dim_a, int32_t dim_b) {
  if (a.shape().size() < 2) throw std::invalid_argument("transpose requires rank >= 2");
  const size_t axis_a = rtensor::normalise_dimension(a.shape().size(), dim_a);
  const size_t axis_b = rtensor::normalise_dimension(a.shape().size(), dim_b);
  if (axis_a == axis_b) throw std::invalid_argument("transpose dimensions must be different");
  if (output.shape() != rtensor::infer_transpose(a.shape(), dim_a, dim_b))
    throw std::invalid_argument("transpose destination has incorrect shape");
  Op &op = impl_->record(Kind::Transpose);
  op.t[0] = ref(a);
  op.t[1] = ref(output);
  op.i0 = static_cast<int32_t>(axis_a);
  op.i1 = static_cast<int32_t>(axis_b);
}

// src/my_metal/runtime.cpp:571-581
void Runtime::split_last_dim(const Mat &a, Mat &output, uint32_t outer, uint32_t inner) {
  if (output.shape() != rtensor::infer_split_last_dim(a.shape(), outer, inner))
    throw std::invalid_argument("split_last_dim destination has incorrect shape");
  Op &op = impl_->record(Kind::Copy);
  op.t[0] = ref(a);
  op.t[1] = ref(output);
}

// src/my_metal/runtime.cpp:583-593
void Runtime::merge_last_dims(const Mat &a, Mat &output, uint32_t outer, uint32_t inner) {
  if (output.shape() != rtensor::infer_merge_last_dims(a.shape(), outer, inner))
    throw std::invalid_argument("merge_last_dims destination has incorrect shape");
  Op &op = impl_->record(Kind::Copy);
  op.t[0] = ref(a);
  op.t[1] = ref(output);
}

// -------------------------------------------------------------- row operators
// src/my_metal/runtime.cpp:747-766
void Runtime::softmax(const Mat &x, Mat &output) {
  if (x.shape().empty() || x.shape().back() == 0)
    throw std::invalid_argument("softmax requires a non-empty final dimension");
  if (output.shape() != x.shape())
    throw std::invalid_argument("softmax destination has incorrect shape");
  Op &op = impl_->record(Kind::Softmax);
  op.t[0] = ref(x);
  op.t[1] = ref(output);
}

namespace {
// src/my_metal/runtime.cpp:768-841 (shared argument checks)
void check_xent(const char *name, const Mat &logits, const IndexMat &targets) {
  const std::string n(name);
  if (logits.shape().size() < 2 || logits.shape().back() == 0)
    throw std::invalid_argument(n + " requires logits with a non-empty final dimension");
  if (targets.shape().size() + 1 != logits.shape().size())
    throw std::invalid_argument(n + " target rank must be one less than logits rank");
  for (size_t i = 0; i < targets.shape().size(); ++i)
    if (targets.shape()[i] != logits.shape()[i])
      throw std::invalid_argument(n + " target shape must match logits leading dimensions");
}
}  // namespace

void Runtime::cross_entropy(const Mat &logits, const IndexMat &targets, Mat &output) {
  check_xent("cross_entropy", logits, targets);
  auto output_shape = targets.shape();
  output_shape.push_back(1);
  if (output.shape() != output_shape)
    throw std::invalid_argument(
        "cross_entropy destination must match target shape with a trailing singleton "
        "dimension");
  Op &op = impl_->record(Kind::Xent);
  op.t[0] = ref(logits);
  op.t[1] = ref(targets);
  op.t[2] = ref(output);
}

void Runtime::cross_entropy_derivative(const Mat &logits, const IndexMat &targets, Mat &output) {
  check_xent("cross_entropy_derivative", logits, targets);
  if (output.shape() != logits.shape())
    throw std::invalid_argument("cross_entropy_derivative destination must match logits shape");
  Op &op = impl_->record(Kind::XentBwd);
  op.t[0] = ref(logits);
  op.t[1] = ref(targets);
  op.t[2] = ref(output);
}

// src/my_metal/runtime.cpp:1031-1059
void Runtime::RMS(const Mat &values, Mat &destination) {
  auto rms_shape = values.shape();
  if (rms_shape.empty()) throw std::invalid_argument("RMS requires a non-empty tensor");
  rms_shape.back() = 1;
  if (destination.shape() != rms_shape)
    throw std::invalid_argument("RMS destination has incorrect shape");
  if (values.shape().back() == 0) throw std::invalid_argument("RMS requires non-empty rows");
  Op &op = impl_->record(Kind::Rms);
  op.t[0] = ref(values);
  op.t[1] = ref(destination);
}

// src/my_metal/runtime.cpp:1061-1072
void Runtime::RMSNorm(const Mat &values, Mat &destination) {
  if (destination.shape() != values.shape())
    throw std::invalid_argument("RMSNorm destination has incorrect shape");
  if (values.shape().empty() || values.shape().back() == 0)
    throw std::invalid_argument("RMSNorm requires non-empty rows");
  Op &op = impl_->record(Kind::RmsNorm);
  op.t[0] = ref(values);
  op.t[1] = ref(destination);
}

// ----------------------------------------------------------------- embedding
// src/my_metal/runtime.cpp:920-944
void Runtime::embedding_lookup(const Mat &weights, const IndexMat &ids, Mat &output) {
  if (weights.shape().size() != 2)
    throw std::invalid_argument("embedding weights must have rank 2");
  auto expected = ids.shape();
  expected.push_back(weights.shape().back());
  if (output.shape() != expected)
    throw std::invalid_argument("embedding output shape does not match IDs");
  Op &op = impl_->record(Kind::Gather);
  op.t[0] = ref(weights);
  op.t[1] = ref(ids);
  op.t[2] = ref(output);
}

// src/my_metal/runtime.cpp:946-950
void Runtime::gather_rows(const Mat &values, const IndexMat &indices, Mat &output) {
  embedding_lookup(values, indices, output);
}

namespace {
// src/my_metal/runtime.cpp:952-981
void check_scatter(const Mat &values, const IndexMat &ids, const Mat &destination) {
  if (destination.shape().size() != 2)
    throw std::invalid_argument("scatter destination must have rank 2");
  auto expected = ids.shape();
  expected.push_back(destination.shape().back());
  if (values.shape() != expected)
    throw std::invalid_argument("scatter input shape does not match IDs and embedding size");
}
}  // namespace

// src/my_metal/runtime.cpp:983-1009
void Runtime::scatter_add_rows(const Mat &base, const IndexMat &ids, const Mat &values,
                               Mat &destination) {
  if (base.shape() != destination.shape())
    throw std::invalid_argument("scatter base and destination shapes must match");
  check_scatter(values, ids, destination);
  Op &op = impl_->record(Kind::Scatter);
  op.t[0] = ref(values);
  op.t[1] = ref(ids);
  op.t[2] = ref(base);
  op.t[3] = ref(destination);
  op.workspace = tl_embedding_scatter_workspace_size(static_cast<uint32_t>(ids.numel()),
                                                     destination.shape()[0],
                                                     destination.shape()[1]);
}

// src/my_metal/runtime.cpp:1011-1030
void Runtime::scatter_index(const Mat &values, const IndexMat &ids, Mat &destination) {
  check_scatter(values, ids, destination);
  Op &op = impl_->record(Kind::Scatter);
  op.t[0] = ref(values);
  op.t[1] = ref(ids);
  op.t[3] = ref(destination);
  op.workspace = tl_embedding_scatter_workspace_size(static_cast<uint32_t>(ids.numel()),
                                                     destination.shape()[0],
                                                     destination.shape()[1]);
}

// ----------------------------------------------------------------- optimiser
// src/my_metal/runtime.cpp:1083-1101
void Runtime::accumulate_gradient_squared_norm(const Mat &gradient, Mat &squared_norm) {
  if (squared_norm.numel() != 1)
    throw std::invalid_argument("gradient norm destination must be a scalar");
  Op &op = impl_->record(Kind::SqNorm);
  op.t[0] = ref(gradient);
  op.t[1] = ref(squared_norm);
  op.workspace = tl_grad_sqnorm_workspace_size(gradient.numel());
}

// src/my_metal/runtime.cpp:1103-1127
void Runtime::clip_gradient(const Mat &gradient, const Mat &squared_norm, kernel_type max_norm,
                            Mat &destination) {
  if (squared_norm.numel() != 1) throw std::invalid_argument("gradient norm input must be a scalar");
  if (gradient.shape() != destination.shape())
    throw std::invalid_argument("gradient clipping input and destination shapes must match");
  if (!(max_norm > 0.0f) || !std::isfinite(max_norm))
    throw std::invalid_argument("maximum gradient norm must be finite and positive");
  Op &op = impl_->record(Kind::Clip);
  op.t[0] = ref(gradient);
  op.t[1] = ref(squared_norm);
  op.t[2] = ref(destination);
  op.f0 = max_norm;
}

// src/my_metal/runtime.cpp:1129-1168
void Runtime::adamW(const Mat &parameter, const Mat &gradient, Mat &destination, Mat &momentum1,
                    Mat &momentum2, const Mat &beta1, const Mat &beta2, const Mat &decay,
                    const Mat &learning_rate, kernel_type epsilon, uint32_t step) {
  if (gradient.shape() != parameter.shape() || destination.shape() != parameter.shape() ||
      momentum1.shape() != parameter.shape() || momentum2.shape() != parameter.shape())
    throw std::invalid_argument("AdamW tensor shapes must match");
  if (beta1.numel() != 1 || beta2.numel() != 1 || decay.numel() != 1 || learning_rate.numel() != 1)
    throw std::invalid_argument("AdamW parameters must be scalars");
  if (step == 0) throw std::invalid_argument("AdamW step must be greater than zero");
  Op &op = impl_->record(Kind::AdamW);
  op.t[0] = ref(parameter);
  op.t[1] = ref(gradient);
  op.t[2] = ref(destination);
  op.t[3] = ref(momentum1);
  op.t[4] = ref(momentum2);
  op.t[5] = ref(beta1);
  op.t[6] = ref(beta2);
  op.t[7] = ref(decay);
  op.t[8] = ref(learning_rate);
  op.f0 = epsilon;
  op.u0 = step;
}

}  // namespace cuda
