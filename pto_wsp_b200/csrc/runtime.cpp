// Run-time half of the cuda_sm100a target: the task loop.
//
// The generated CPU-sim `<module>_main` walks the workload tree and, per task,
// builds a KernelTaskDesc, calls the kernel synchronously and feeds its cycle
// charge to a makespan scheduler (src/python/pto_codegen.cpp:2245-2697).  Here
// the same walk *enqueues* tasks instead of running them: each task becomes a
// record of the device task table (view offsets, axis args, scalar args) and
// is placed in the current dependency wave.  A wave closes when a task touches
// a tile that an earlier task of the wave writes (or writes one it reads), so
// everything inside a wave runs concurrently and waves run in program order --
// the same results as the sequential CPU-sim.  The reference scheduler model
// (Scheduler::issue, :1562-1606) runs alongside, so the returned makespan is
// the CPU-sim's own u64.
//
// Workloads without data-dependent control flow (no cond / select / slots)
// are walked once per distinct set of run-time sizes; later runs replay the
// cached waves and task table straight from device memory.
#include <cuda_runtime_api.h>

#include <algorithm>
#include <climits>
#include <chrono>
#include <fstream>
#include <functional>
#include <unordered_map>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <queue>
#include <sstream>
#include <unordered_set>

#include "jit.hpp"
#include "runtime.hpp"

namespace ptowsp {

uint64_t reference_kernel_cycles(const KernelDef& kd);

namespace {

thread_local std::string g_err;

#define PW_CUDA(call)                                                                              \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess)                                                                     \
            throw Error(PTOWSP_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));     \
    } while (0)

// The reference makespan model (Scheduler::issue, pto_codegen.cpp:1562-1606).
struct Scheduler {
    uint32_t n;
    uint64_t window;
    uint64_t issue_time = 0;
    std::vector<uint64_t> avail;
    std::priority_queue<uint64_t, std::vector<uint64_t>, std::greater<uint64_t>> in_flight;
    Scheduler(uint32_t workers, uint64_t w) : n(workers ? workers : 1), window(w), avail(n, 0) {}
    void advance_to(uint64_t t) {
        if (t > issue_time) issue_time = t;
        while (!in_flight.empty() && in_flight.top() <= issue_time) in_flight.pop();
    }
    uint64_t issue(uint64_t dur, uint32_t wid, uint64_t ready) {
        if (wid >= n) wid = 0;
        advance_to(ready);
        if (window > 0)
            while (in_flight.size() >= window) advance_to(in_flight.top());
        const uint64_t start = avail[wid] > issue_time ? avail[wid] : issue_time;
        const uint64_t end = start + dur;
        avail[wid] = end;
        in_flight.push(end);
        return end;
    }
};

struct Val {
    Expr::Ty ty;
    uint64_t v;
};

int64_t as_i64(uint64_t v) { return static_cast<int64_t>(v); }

// FNV-1a over a CSR selection's indptr[0..outer] and indices[0..indptr[outer]) (the arrays a Select walk reads).
uint64_t csr_hash(const int32_t* indptr, const int32_t* indices, int64_t outer) {
    uint64_t h = 1469598103934665603ull;
    auto mix = [&](int32_t v) {
        for (int k = 0; k < 4; ++k) {
            h ^= static_cast<uint64_t>((static_cast<uint32_t>(v) >> (8 * k)) & 0xffu);
            h *= 1099511628211ull;
        }
    };
    if (!indptr || outer < 0) return h;
    for (int64_t i = 0; i <= outer; ++i) mix(indptr[i]);
    const int64_t nnz = indptr[outer];
    for (int64_t p = 0; indices && p < nnz; ++p) mix(indices[p]);
    return h;
}

dev::ParamType ptype(DType d) {
    switch (d) {
        case DType::F32: return dev::PT_F32;
        case DType::F16: return dev::PT_F16;
        case DType::I32: return dev::PT_I32;
        case DType::U32: return dev::PT_U32;
        case DType::I64: return dev::PT_I64;
        case DType::U64: return dev::PT_U64;
        default: return dev::PT_OTHER;
    }
}

struct Walker {
    Program& P;
    RuntimeContext* ctx;
    std::vector<TensorBinding>& T;
    LaunchProgram& L;
    std::vector<std::pair<const std::string*, int64_t>> env;  // loop var -> value
    Scheduler sched;
    uint64_t rr = 0;
    // Dependency levels: a task goes to the first wave after the last wave that
    // wrote a tile it touches, or read a tile it writes (RAW, WAR, WAW).
    std::unordered_map<uint64_t, size_t> last_write, max_read;
    size_t wave_floor = 0;  // waves below this were launched by a flush
    std::vector<std::string>& log;
    std::function<void()> flush;
    bool dry = false;
    std::vector<uint8_t> written_any;  // tensors written by a task so far
    // host copies of device tensors read by slot_load_u64 that no task of this run has written (yet): one
    // device-to-host copy serves every slot load from that tensor instead of a synchronising read per load
    std::vector<std::vector<unsigned char>> slot_mirror;
    static constexpr size_t kSlotMirrorMax = size_t(64) << 20;
    // full-overwrite tracking: elements stored per tensor and whether any two stores hit the same tile
    std::vector<int64_t> write_elems;
    std::vector<std::unordered_set<uint64_t>> write_keys;
    std::vector<uint8_t> write_partial;
    bool fully_written(size_t tid) const {
        int64_t numel = 1;
        for (auto d : P.plan.tensors[tid].shape) numel *= d;
        return written_any[tid] && !write_partial[tid] && write_elems[tid] == numel;
    }

    // ---- a pipeline body as device processes: per-process operations, checked as the walk goes ----
    struct CspCapture {
        int nproc = 0, cur = -1;
        bool ok = true;
        std::string why;
        std::vector<std::vector<dev::CspOp>> ops;      // per process
        std::vector<int64_t> rec;
        std::unordered_map<const Node*, int> slot_of;
        std::vector<const Node*> slot_node;
        std::vector<int> sender, receiver;             // per channel: its one sending / receiving process
        std::vector<int32_t> cap;                      // per channel: device capacity
        std::vector<std::vector<uint32_t>> vc;         // per process: tasks of each process ordered before this point
        std::vector<std::vector<std::vector<uint32_t>>> sent_vc, recv_vc;  // per channel: clock at each send / receive
        struct Access {
            int proc;
            uint32_t idx;
        };
        std::unordered_map<uint64_t, Access> last_w;
        std::unordered_map<uint64_t, std::vector<Access>> readers;  // since the last write
        uint64_t checks = 0;
        void fail(const std::string& w) {
            if (ok) why = w;
            ok = false;
        }
        bool ordered(const Access& a, int p) const { return a.proc == p || vc[p][a.proc] > a.idx; }
    };
    std::unique_ptr<CspCapture> csp;

    void csp_task(const Node& n, const Batch& b, const uint64_t* rkeys, int nr, const uint64_t* wkeys, int nw) {
        CspCapture& C = *csp;
        if (!C.ok || C.cur < 0) return;
        const int p = C.cur;
        const KernelImpl& ki = P.impls[n.kernel_index];
        if (!ki.tp_ok) return C.fail("kernel '" + P.plan.kernels[n.kernel_index].name + "' has no interpreter program");
        if (extra_read_key) return C.fail("a task reads a device-selected condition");
        const uint32_t idx = C.vc[p][p];
        constexpr uint64_t kMaxChecks = 20000000;
        for (int i = 0; i < nr; ++i) {
            if (auto f = C.last_w.find(rkeys[i]); f != C.last_w.end() && !C.ordered(f->second, p))
                return C.fail("a read is not ordered after another process's write by the channels");
            C.readers[rkeys[i]].push_back({p, idx});
        }
        for (int i = 0; i < nw; ++i) {
            if (auto f = C.last_w.find(wkeys[i]); f != C.last_w.end() && !C.ordered(f->second, p))
                return C.fail("two processes write a tile in an order the channels do not fix");
            auto& rd = C.readers[wkeys[i]];
            C.checks += rd.size();
            for (const auto& a : rd)
                if (!C.ordered(a, p)) return C.fail("a write is not ordered after another process's read by the channels");
            rd.clear();
            C.last_w[wkeys[i]] = {p, idx};
        }
        if (C.checks > kMaxChecks) return C.fail("too many hazards to check");
        auto [it, fresh] = C.slot_of.emplace(&n, static_cast<int>(C.slot_node.size()));
        if (fresh) C.slot_node.push_back(&n);
        const size_t words = static_cast<size_t>(b.stride);
        dev::CspOp op{dev::CSP_TASK, it->second, static_cast<int64_t>(C.rec.size())};
        C.rec.insert(C.rec.end(), b.rec.end() - static_cast<std::ptrdiff_t>(words), b.rec.end());
        C.ops[p].push_back(op);
        C.vc[p][p]++;
    }
    void csp_channel(int c, bool send) {
        CspCapture& C = *csp;
        if (!C.ok || C.cur < 0) return;
        const int p = C.cur;
        int& who = send ? C.sender[c] : C.receiver[c];
        if (who >= 0 && who != p) return C.fail("a channel with more than one " + std::string(send ? "sender" : "receiver"));
        who = p;
        auto join = [&](const std::vector<uint32_t>& o) {
            for (int q = 0; q < C.nproc; ++q) C.vc[p][q] = std::max(C.vc[p][q], o[q]);
        };
        if (send) {
            const size_t k = C.sent_vc[c].size();  // a send waits for the receive cap tokens before it
            if (k >= static_cast<size_t>(C.cap[c])) {
                if (C.recv_vc[c].size() <= k - C.cap[c]) return C.fail("a send runs ahead of its channel's receives");
                join(C.recv_vc[c][k - C.cap[c]]);
            }
            C.sent_vc[c].push_back(C.vc[p]);
        } else {
            const size_t k = C.recv_vc[c].size();  // a receive waits for its send
            if (C.sent_vc[c].size() <= k) return C.fail("a receive without its send");
            join(C.sent_vc[c][k]);
            C.recv_vc[c].push_back(C.vc[p]);
        }
        C.ops[p].push_back(dev::CspOp{send ? dev::CSP_SEND : dev::CSP_RECV, c, 0});
    }

    Walker(Program& p, RuntimeContext* c, std::vector<TensorBinding>& t, LaunchProgram& l, std::vector<std::string>& lg)
        : P(p), ctx(c), T(t), L(l),
          sched(static_cast<uint32_t>(p.plan.schedule.num_targets > 0 ? p.plan.schedule.num_targets
                                      : (p.plan.schedule.streams > 0 ? p.plan.schedule.streams : 1)),
                static_cast<uint64_t>(p.plan.schedule.window_tasks)),
          log(lg) {
        written_any.assign(p.plan.tensors.size(), 0);
        slot_mirror.resize(p.plan.tensors.size());
        write_elems.assign(p.plan.tensors.size(), 0);
        write_keys.resize(p.plan.tensors.size());
        write_partial.assign(p.plan.tensors.size(), 0);
    }

    int64_t var(const std::string& name) const {
        for (auto it = env.rbegin(); it != env.rend(); ++it)
            if (*it->first == name) return it->second;
        throw Error(PTOWSP_ERR_PLAN, "loop variable '" + name + "' is not in scope");
    }
    bool var_by_id(uint64_t id, int64_t& out) const {
        for (auto it = env.rbegin(); it != env.rend(); ++it)
            if (fnv1a_64(*it->first) == id) {
                out = it->second;
                return true;
            }
        return false;
    }

    std::unordered_set<std::string> seen;
    void note(std::string q) {
        if (seen.insert(q).second) log.push_back(std::move(q));
    }
    // loops over a ragged axis or a selection whose body is one task (candidates for device-side expansion)
    struct LoopNote {
        const Node* node;
        char kind;
        std::string key_name;
        std::vector<int64_t> vars;  // selection: the loop variable of each iteration
    };
    std::vector<LoopNote> loops;
    uint64_t symbol_u64(uint64_t id) {
        uint64_t v = ctx->get_symbol_u64 ? ctx->get_symbol_u64(ctx->ctx, id) : 0;
        note("s" + std::to_string(id) + "=" + std::to_string(v));
        return v;
    }
    int64_t axis_size(const std::string& name) {
        int64_t v = ctx->get_axis_size ? ctx->get_axis_size(ctx->ctx, name.c_str()) : 0;
        note("a" + name + "=" + std::to_string(v));
        return v;
    }
    uint64_t slot(uint32_t i) { return ctx->get_slot_u64 ? ctx->get_slot_u64(ctx->ctx, i) : 0; }

    Val eval(const Expr& e, const std::vector<uint64_t>* task_args) {
        switch (e.op) {
            case Expr::Op::Lit: return {e.ty, e.v};
            case Expr::Op::Axis: {
                int64_t v;
                if (!var_by_id(e.v, v)) throw Error(PTOWSP_ERR_PLAN, "emit_scalar_expr_cpp: axis_var not in scope");
                return {Expr::Ty::I64, static_cast<uint64_t>(v)};
            }
            case Expr::Op::Sym:
            case Expr::Op::Tag: return {Expr::Ty::U64, symbol_u64(e.v)};
            case Expr::Op::Slot: {
                uint64_t v = slot(static_cast<uint32_t>(e.v));
                if (e.ty == Expr::Ty::Bool) return {Expr::Ty::Bool, v != 0 ? 1ull : 0ull};
                return {e.ty, v};
            }
            case Expr::Op::TaskParam: {
                if (!task_args) throw Error(PTOWSP_ERR_PLAN, "task_param() outside a task");
                return {Expr::Ty::U64, e.v < task_args->size() ? (*task_args)[e.v] : 0ull};
            }
            case Expr::Op::Unary: {
                Val a = eval(*e.a, task_args);
                if (e.fn == "!") return {Expr::Ty::Bool, a.v == 0 ? 1ull : 0ull};
                if (e.fn == "-") return {a.ty == Expr::Ty::U64 ? Expr::Ty::U64 : Expr::Ty::I64, ~a.v + 1};
                return {a.ty == Expr::Ty::U64 ? Expr::Ty::U64 : Expr::Ty::I64, ~a.v};
            }
            case Expr::Op::Ternary: {
                Val c = eval(*e.c, task_args);
                return c.v ? eval(*e.a, task_args) : eval(*e.b, task_args);
            }
            case Expr::Op::Cast: {
                Val a = eval(*e.a, task_args);
                if (e.ty == Expr::Ty::Bool) return {Expr::Ty::Bool, a.v != 0 ? 1ull : 0ull};
                return {e.ty, a.v};
            }
            case Expr::Op::Binary: {
                Val a = eval(*e.a, task_args);
                Val b = eval(*e.b, task_args);
                const std::string& f = e.fn;
                if (f == "&&") return {Expr::Ty::Bool, (a.v && b.v) ? 1ull : 0ull};
                if (f == "||") return {Expr::Ty::Bool, (a.v || b.v) ? 1ull : 0ull};
                const bool u = a.ty == Expr::Ty::U64 || b.ty == Expr::Ty::U64;  // usual arithmetic conversions
                const Expr::Ty rt = u ? Expr::Ty::U64 : Expr::Ty::I64;
                auto cmp = [&](auto op) -> Val {
                    bool r = u ? op(a.v, b.v) : op(as_i64(a.v), as_i64(b.v));
                    return {Expr::Ty::Bool, r ? 1ull : 0ull};
                };
                if (f == "<") return cmp([](auto x, auto y) { return x < y; });
                if (f == "<=") return cmp([](auto x, auto y) { return x <= y; });
                if (f == ">") return cmp([](auto x, auto y) { return x > y; });
                if (f == ">=") return cmp([](auto x, auto y) { return x >= y; });
                if (f == "==") return cmp([](auto x, auto y) { return x == y; });
                if (f == "!=") return cmp([](auto x, auto y) { return x != y; });
                uint64_t r = 0;
                if (f == "+") r = a.v + b.v;
                else if (f == "-") r = a.v - b.v;
                else if (f == "*") r = a.v * b.v;
                else if (f == "/") {
                    if (b.v == 0) throw Error(PTOWSP_ERR_ARG, "scalar expression divides by zero");
                    r = u ? a.v / b.v : static_cast<uint64_t>(as_i64(a.v) / as_i64(b.v));
                } else if (f == "%") {
                    if (b.v == 0) throw Error(PTOWSP_ERR_ARG, "scalar expression divides by zero");
                    r = u ? a.v % b.v : static_cast<uint64_t>(as_i64(a.v) % as_i64(b.v));
                } else if (f == "&") r = a.v & b.v;
                else if (f == "|") r = a.v | b.v;
                else if (f == "^") r = a.v ^ b.v;
                else if (f == "<<") r = a.v << (b.v & 63);
                else if (f == ">>") r = u ? (a.v >> (b.v & 63)) : static_cast<uint64_t>(as_i64(a.v) >> (b.v & 63));
                else throw Error(PTOWSP_ERR_PLAN, "unknown scalar operator " + f);
                return {rt, r};
            }
        }
        return {Expr::Ty::U64, 0};
    }

    uint64_t arg_value(const ArgSpec& a) {
        switch (a.kind) {
            case ArgSpec::Kind::Var: return static_cast<uint64_t>(var(a.var));
            case ArgSpec::Kind::Sym: return symbol_u64(a.v);
            default: return a.v;
        }
    }

    // view offset (elements) of a tensor arg at the current loop values
    int64_t view_offset(const TensorArg& ta) {
        const auto& st = T[ta.tensor].strides;
        int64_t off = 0;
        for (size_t d = 0; d < ta.index.size(); ++d) {
            int64_t v = ta.index[d].is_var ? var(ta.index[d].var) : ta.index[d].c;
            off += v * (d < st.size() ? st[d] : 0);
        }
        return off;
    }

    static uint64_t mix64(uint64_t z) {  // splitmix64 finaliser
        z += 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    }
    // Tile key: tensor id + the view's leading indices, cut to the coarsest
    // index depth any view of that tensor uses (so views at different depths
    // that overlap get the same key).
    uint64_t view_key(const TensorArg& ta) {
        int depth = std::max(P.tensor_key_depth[ta.tensor], 0);
        uint64_t h = mix64(0x51ED27A0ull + ta.tensor);
        for (int d = 0; d < depth && d < static_cast<int>(ta.index.size()); ++d) {
            int64_t v = ta.index[d].is_var ? var(ta.index[d].var) : ta.index[d].c;
            h = mix64(h ^ (static_cast<uint64_t>(v) * 0xD6E8FEB86659FD93ull + static_cast<uint64_t>(d)));
        }
        return h;
    }

    // After a flush every later task must land in a wave that was not launched yet.
    void close_wave() {
        while (!L.waves.empty() && L.waves.back().batches.empty()) L.waves.pop_back();
        wave_floor = L.waves.size();
    }

    uint64_t node(const Node& n, uint64_t ready) {
        switch (n.kind) {
            case Node::Kind::SlotSet:
                if (ctx->set_slot_u64) ctx->set_slot_u64(ctx->ctx, n.slot, n.slot_value);
                return ready;
            case Node::Kind::SlotLoad: {
                const TensorArg& ta = n.slot_tensor;
                const TensorBinding& tb = T[ta.tensor];
                const int64_t base = view_offset(ta);
                int64_t s3 = 0, s4 = 1;
                if (ta.view_rank >= 2) {
                    s3 = tb.strides[ta.base_rank - ta.view_rank];
                    s4 = tb.strides[ta.base_rank - ta.view_rank + 1];
                } else if (ta.view_rank == 1) {
                    s4 = tb.strides[ta.base_rank - 1];
                }
                const int64_t off = base + n.row * s3 + n.col * s4;
                if (off < 0 || off >= tb.span) throw Error(PTOWSP_ERR_ARG, "slot_load_u64 reads outside its tensor");
                if (n.dev_deferred) {  // the cond tree after it is decided on the GPU from this element
                    deferred_off = off;
                    return ready;
                }
                const DType dt = P.plan.tensors[ta.tensor].dtype;
                const int eb = dtype_bytes(dt);
                alignas(8) unsigned char buf[8] = {0};
                if (!dry && tb.on_device && !written_any[ta.tensor] && tb.bytes <= kSlotMirrorMax) {
                    // device input that no enqueued task writes: no wave has to finish before reading it
                    std::vector<unsigned char>& m = slot_mirror[ta.tensor];
                    if (m.empty()) {
                        m.resize(tb.bytes);
                        PW_CUDA(cudaMemcpy(m.data(), tb.dev, tb.bytes, cudaMemcpyDeviceToHost));
                        ++P.timing.slot_syncs;
                    }
                    std::memcpy(buf, m.data() + off * eb, eb);
                } else if (!dry && (tb.on_device || written_any[ta.tensor])) {
                    flush();  // data written by enqueued tasks: finish the waves, then read the element back
                    PW_CUDA(cudaMemcpy(buf, tb.dev + off * eb, eb, cudaMemcpyDeviceToHost));
                    ++P.timing.slot_syncs;
                } else {
                    std::memcpy(buf, static_cast<const char*>(tb.user_ptr) + off * eb, eb);
                }
                uint64_t v = 0;
                switch (dt) {  // (uint64_t)((item*)ptr)[...] of the emitted code
                    case DType::F32: { float f; std::memcpy(&f, buf, 4); v = static_cast<uint64_t>(static_cast<int64_t>(f)); break; }
                    case DType::F64: { double f; std::memcpy(&f, buf, 8); v = static_cast<uint64_t>(static_cast<int64_t>(f)); break; }
                    case DType::I32: { int32_t x; std::memcpy(&x, buf, 4); v = static_cast<uint64_t>(static_cast<int64_t>(x)); break; }
                    case DType::U32: { uint32_t x; std::memcpy(&x, buf, 4); v = x; break; }
                    case DType::I64: case DType::U64: std::memcpy(&v, buf, 8); break;
                    case DType::I16: { int16_t x; std::memcpy(&x, buf, 2); v = static_cast<uint64_t>(static_cast<int64_t>(x)); break; }
                    case DType::U16: { uint16_t x; std::memcpy(&x, buf, 2); v = x; break; }
                    case DType::I8: { int8_t x; std::memcpy(&x, buf, 1); v = static_cast<uint64_t>(static_cast<int64_t>(x)); break; }
                    case DType::U8: case DType::Bool: v = buf[0]; break;
                    default: throw Error(PTOWSP_ERR_UNSUPPORTED, "slot_load_u64 from this dtype");
                }
                if (ctx->set_slot_u64) ctx->set_slot_u64(ctx->ctx, n.slot, v);
                return ready;
            }
            case Node::Kind::ParallelFor:
            case Node::Kind::ForEach: {
                int64_t ub = 0;
                if (n.axis.kind == Axis::Kind::Dense) {
                    ub = n.axis.size;
                } else if (n.axis.kind == Axis::Kind::DenseDyn) {
                    ub = axis_size(n.var);
                } else {
                    int64_t outer = static_cast<int64_t>(symbol_u64(n.axis.outer_sym));
                    const int32_t* lens = ctx->get_symbol_ptr
                                              ? static_cast<const int32_t*>(ctx->get_symbol_ptr(ctx->ctx, n.axis.lengths_sym))
                                              : nullptr;
                    if (lens)
                        for (int64_t i = 0; i < outer; ++i) ub += lens[i];
                    const std::string kn = "r" + std::to_string(n.axis.lengths_sym) + ":" + std::to_string(n.axis.outer_sym);
                    note(kn + "=" + std::to_string(ub));
                    if (n.body && n.body->kind == Node::Kind::Task) loops.push_back({&n, 'r', kn, {}});
                }
                uint64_t done = ready, cur = ready;
                env.push_back({&n.var, 0});
                for (int64_t i = 0; i < ub; ++i) {
                    env.back().second = i;
                    if (n.kind == Node::Kind::ParallelFor) done = std::max(done, node(*n.body, ready));
                    else cur = node(*n.body, cur);
                }
                env.pop_back();
                return n.kind == Node::Kind::ParallelFor ? done : cur;
            }
            case Node::Kind::Select: {
                int64_t outer = static_cast<int64_t>(symbol_u64(n.outer_sym));
                const int32_t* indptr = ctx->get_symbol_ptr ? static_cast<const int32_t*>(ctx->get_symbol_ptr(ctx->ctx, n.indptr_sym)) : nullptr;
                const int32_t* indices = ctx->get_symbol_ptr ? static_cast<const int32_t*>(ctx->get_symbol_ptr(ctx->ctx, n.indices_sym)) : nullptr;
                int64_t nnz = indptr ? indptr[outer] : 0;
                // the walk depends on the CSR arrays themselves: key a cached task table on their contents
                const std::string kn = "c" + std::to_string(n.indptr_sym) + ":" + std::to_string(n.indices_sym) + ":" +
                                       std::to_string(n.outer_sym);
                note(kn + "=" + std::to_string(csr_hash(indptr, indices, outer)));
                if (n.body && n.body->kind == Node::Kind::Task) {
                    loops.push_back({&n, 'c', kn, {}});
                    for (int64_t p = 0; p < nnz; ++p) loops.back().vars.push_back(indices ? indices[p] : 0);
                }
                uint64_t done = ready;
                env.push_back({&n.var, 0});
                for (int64_t p = 0; p < nnz; ++p) {
                    env.back().second = indices ? indices[p] : 0;
                    done = std::max(done, node(*n.body, ready));
                }
                env.pop_back();
                return done;
            }
            case Node::Kind::Cond: {
                if (n.dev_select) return dev_select(*n.dev_select, ready);
                Val c = eval(*n.pred, nullptr);
                return node(c.v ? *n.then_n : *n.else_n, ready);
            }
            case Node::Kind::Combine: {
                uint64_t done = ready;
                for (auto& ch : n.children) done = std::max(done, node(*ch, ready));
                return done;
            }
            case Node::Kind::Sequential: {
                uint64_t cur = ready;
                for (auto& ch : n.children) cur = node(*ch, cur);
                return cur;
            }
            case Node::Kind::Task: return task(n, ready);
            case Node::Kind::Pipeline: return std::max(ready, pipeline(n));
            case Node::Kind::Send:
            case Node::Kind::Consume:
                throw Error(PTOWSP_ERR_PLAN, "send / consume outside a CSP pipeline process");
        }
        return ready;
    }

    uint64_t task(const Node& n, uint64_t ready) {
        std::vector<uint64_t> args = enqueue(n);
        const KernelImpl& ki = P.impls[n.kernel_index];
        // worker choice + makespan (pto_codegen.cpp:2679-2692)
        const Schedule& sc = P.plan.schedule;
        uint32_t wid = 0;
        if (!sc.dispatch_policy.empty()) {
            if (sc.dispatch_policy == "round_robin" || sc.dispatch_policy == "work_steal") {
                wid = static_cast<uint32_t>(rr++ % sched.n);
            } else {
                Val key = eval(*sc.dispatch_key, &args);
                wid = static_cast<uint32_t>(key.v % sched.n);
            }
        }
        return sched.issue(ki.cycles, wid, ready);
    }

    // One task whose scalars the GPU picks (dev_select): the template leaf is placed once, reading the slot's
    // tensor element as well; its batch gets a row [task, element, signed mask, operands, leaf scalars].
    int64_t deferred_off = -1;
    Batch* last_batch = nullptr;
    uint64_t dev_select(const DevSelect& ds, uint64_t ready) {
        if (deferred_off < 0) throw Error(PTOWSP_ERR_PLAN, "device-selected cond without its slot load");
        const int nc = static_cast<int>(ds.cmp.size());
        const Node& leaf = *ds.leaves[0];
        const TensorArg& st = ds.load->slot_tensor;
        extra_read_key = view_key(st);
        const uint64_t done = task(leaf, ready);
        extra_read_key = 0;
        Batch& b = *last_batch;
        const int nscal = static_cast<int>(leaf.scalar_args.size());
        const int words = 3 + nc + static_cast<int>(ds.leaves.size()) * nscal;
        if (b.sel && (b.sel != &ds || b.sel_row_words != words))
            throw Error(PTOWSP_ERR_PLAN, "one task node under two device-selected conds");
        b.sel = &ds;
        b.sel_tensor = st.tensor;
        b.sel_row_words = words;
        uint64_t mask = 0;
        std::vector<uint64_t> row;
        row.reserve(words);
        row.push_back(static_cast<uint64_t>(b.ntasks - 1));
        row.push_back(static_cast<uint64_t>(deferred_off));
        row.push_back(0);
        for (int c = 0; c < nc; ++c) {
            const Val o = eval(*ds.other[c], nullptr);
            if (ds.slot_expr[c]->ty != Expr::Ty::U64 && o.ty != Expr::Ty::U64) mask |= 1ull << c;  // signed compare
            row.push_back(o.v);
        }
        if (nc > 64) throw Error(PTOWSP_ERR_LIMIT, "device-selected cond tree deeper than 64");
        row[2] = mask;
        for (const Node* lf : ds.leaves)
            for (const auto& a : lf->scalar_args) row.push_back(arg_value(a));
        b.sel_rows.insert(b.sel_rows.end(), row.begin(), row.end());
        deferred_off = -1;
        return done;
    }
    uint64_t extra_read_key = 0;

    // Places one task in its dependency wave; returns its u64 args.
    std::vector<uint64_t> enqueue(const Node& n) {
        const KernelDef& kd = P.plan.kernels[n.kernel_index];
        const KernelImpl& ki = P.impls[n.kernel_index];
        // u64 args: axis args, (valid_row, valid_col) per tensor param, scalar args (pto_codegen.cpp:2526-2545)
        std::vector<uint64_t> args;
        args.reserve(n.axis_args.size() + 2 * kd.num_tensor_params + n.scalar_args.size());
        for (const auto& a : n.axis_args) args.push_back(arg_value(a));
        for (const auto& p : kd.params)
            if (p.tensor_index >= 0) {
                args.push_back(static_cast<uint64_t>(p.v.rows));
                args.push_back(static_cast<uint64_t>(p.v.cols));
            }
        std::vector<uint64_t> scal;
        for (const auto& a : n.scalar_args) scal.push_back(arg_value(a));
        args.insert(args.end(), scal.begin(), scal.end());

        // dependency level
        uint64_t rkeys[dev::kMaxParams + 1], wkeys[dev::kMaxParams];
        int nr = 0, nw = 0;
        size_t level = wave_floor;
        for (int ti = 0; ti < kd.num_tensor_params; ++ti) {
            const TensorArg& ta = n.tensor_args[n.param_to_arg[ti]];
            uint64_t key = view_key(ta);
            if (ki.param_write[ti]) {
                wkeys[nw++] = key;
                if (auto f = last_write.find(key); f != last_write.end()) level = std::max(level, f->second + 1);
                if (auto f = max_read.find(key); f != max_read.end()) level = std::max(level, f->second + 1);
            }
            if (ki.param_read[ti]) {
                rkeys[nr++] = key;
                if (auto f = last_write.find(key); f != last_write.end()) level = std::max(level, f->second + 1);
            }
        }
        if (extra_read_key) {  // the tensor element a device-selected cond reads
            rkeys[nr++] = extra_read_key;
            if (auto f = last_write.find(extra_read_key); f != last_write.end()) level = std::max(level, f->second + 1);
        }
        for (int i = 0; i < nw; ++i) last_write[wkeys[i]] = level;
        for (int i = 0; i < nr; ++i) {
            auto& m = max_read[rkeys[i]];
            m = std::max(m, level);
        }
        while (L.waves.size() <= level) L.waves.emplace_back();

        Wave& w = L.waves[level];
        auto it = w.by_node.find(&n);
        if (it == w.by_node.end()) {
            Batch b;
            b.kernel = n.kernel_index;
            b.node = &n;
            b.stride = kd.num_tensor_params + static_cast<int>(n.axis_args.size()) + kd.num_scalar_params;
            w.batches.push_back(std::move(b));
            it = w.by_node.emplace(&n, w.batches.size() - 1).first;
        }
        Batch& b = w.batches[it->second];
        for (int ti = 0; ti < kd.num_tensor_params; ++ti) {
            const TensorArg& ta = n.tensor_args[n.param_to_arg[ti]];
            const int64_t off = view_offset(ta);
            b.rec.push_back(off);
            if ((off & 3) != 0) b.aligned_rows = false;
            if (ki.param_write[ti]) {
                written_any[ta.tensor] = 1;
                // a store covers its whole view block when the tile has exactly the block's size
                const auto& shape = P.plan.tensors[ta.tensor].shape;
                int64_t block = 1;
                for (size_t d = ta.index.size(); d < shape.size(); ++d) block *= shape[d];
                const KernelParam* kp = nullptr;
                for (const auto& p : kd.params)
                    if (p.tensor_index == ti) kp = &p;
                const bool exact = kp && static_cast<int64_t>(kp->v.rows) * kp->v.cols == block &&
                                   static_cast<int>(ta.index.size()) == P.tensor_key_depth[ta.tensor];
                if (!exact || !write_keys[ta.tensor].insert(view_key(ta)).second) write_partial[ta.tensor] = 1;
                else write_elems[ta.tensor] += block;
            }
        }
        for (size_t i = 0; i < n.axis_args.size(); ++i) b.rec.push_back(static_cast<int64_t>(args[i]));
        for (uint64_t s : scal) b.rec.push_back(static_cast<int64_t>(s));
        b.ntasks++;
        L.tasks++;
        last_batch = &b;
        if (csp) csp_task(n, b, rkeys, nr, wkeys, nw);
        return args;
    }

    // ---- CSP pipelines (CSPT time semantics, pto_codegen.cpp:1611-1705 and :1759-2220) ----
    //
    // Every process keeps its own clock; a task adds its kernel's cycle charge to the clock of the process that
    // runs it; channels carry (token, send time) and a receive moves the receiver's clock to at least send time +
    // channel latency; a sender that had to wait for room moves its clock to at least the time of the last
    // receive.  The result is the largest process clock.  The reference runs each process on its own thread; here
    // the processes are interleaved deterministically on the host: the first runnable process in declaration
    // order runs until its next channel operation completes or blocks (a producer released by a receive runs
    // before the receiver goes on, as a woken thread would), and every task it reaches is placed in the
    // dependency waves in that order, so the GPU runs the tasks in an order the channels allow.
    struct Chan {
        int64_t cap = 0;
        std::deque<std::pair<uint64_t, uint64_t>> buf;  // (token, send time)
        bool closed = false, receiver_waiting = false, has_rdv = false;
        std::pair<uint64_t, uint64_t> rdv{0, 0};
        uint64_t last_pop = 0;
    };
    struct Frame {
        const Node* node;
        int64_t i = 0, ub = 0;
        int state = 0;
    };
    struct Proc {
        std::vector<Frame> stack;
        std::vector<std::pair<const std::string*, int64_t>> env;
        uint64_t t = 0, token = 0;
        bool done = false, blocked = false, resumed = false;
        int wait_send = -1, wait_recv = -1;  // channel this process waits on, as sender / receiver
    };
    enum class Step { Yield, Blocked, Done };

    uint64_t pipeline(const Node& n) {
        const uint64_t latency = symbol_u64(fnv1a_64("__pto_wsp_channel_latency_cycles"));
        std::vector<Chan> ch(n.channels.size());
        for (size_t c = 0; c < ch.size(); ++c) ch[c].cap = n.channels[c].capacity;
        std::vector<Proc> pr(n.processes.size());
        if (&n == P.plan.body.get() && P.opt_csp_device && P.cacheable) {  // the whole body: a device-process candidate
            csp = std::make_unique<CspCapture>();
            CspCapture& C = *csp;
            C.nproc = static_cast<int>(pr.size());
            C.ops.resize(pr.size());
            C.vc.assign(pr.size(), std::vector<uint32_t>(pr.size(), 0));
            C.sender.assign(ch.size(), -1);
            C.receiver.assign(ch.size(), -1);
            C.sent_vc.resize(ch.size());
            C.recv_vc.resize(ch.size());
            for (size_t c = 0; c < ch.size(); ++c)
                C.cap.push_back(static_cast<int32_t>(std::max<int64_t>(1, std::min<int64_t>(n.channels[c].capacity, 1 << 30))));
        }
        for (size_t p = 0; p < pr.size(); ++p) pr[p].stack.push_back(Frame{n.children[p].get()});
        auto wake_senders = [&](int c) {
            for (auto& q : pr)
                if (q.blocked && q.wait_send == c) q.blocked = false, q.resumed = true;
        };
        auto wake_receivers = [&](int c) {
            for (auto& q : pr)
                if (q.blocked && q.wait_recv == c) q.blocked = false, q.resumed = true;
        };
        auto saved = std::move(env);
        for (;;) {
            size_t pick = pr.size();
            for (size_t p = 0; p < pr.size(); ++p)
                if (!pr[p].done && !pr[p].blocked) {
                    pick = p;
                    break;
                }
            if (pick == pr.size()) {
                bool all = true;
                for (auto& q : pr) all = all && q.done;
                if (all) break;
                env = std::move(saved);
                throw Error(PTOWSP_ERR_PLAN, "CSP pipeline deadlock: every unfinished process waits on a channel");
            }
            Proc& p = pr[pick];
            env = std::move(p.env);
            if (csp) csp->cur = static_cast<int>(pick);
            const Step st = step(p, ch, latency, wake_senders, wake_receivers);
            if (csp) csp->cur = -1;
            p.env = std::move(env);
            if (st == Step::Done) {
                p.done = true;
                for (int c : n.processes[pick].produces) {  // close what this process produces
                    ch[c].closed = true;
                    wake_senders(c);
                    wake_receivers(c);
                }
            }
        }
        env = std::move(saved);
        if (csp) {
            CspCapture& C = *csp;
            if (C.ok) {
                auto D = std::make_unique<CspDevice>();
                for (auto& ops : C.ops) {
                    D->proc_first.push_back(static_cast<int32_t>(D->ops.size()));
                    D->ops.insert(D->ops.end(), ops.begin(), ops.end());
                }
                D->proc_first.push_back(static_cast<int32_t>(D->ops.size()));
                D->rec = std::move(C.rec);
                D->slot_node = C.slot_node;
                D->caps = C.cap;
                for (const Node* sn : D->slot_node) D->smem = std::max(D->smem, P.impls[sn->kernel_index].tp_smem);
                L.csp = std::move(D);
                L.csp_note.clear();
            } else {
                L.csp_note = C.why;
            }
            csp.reset();
        }
        uint64_t makespan = 0;
        for (auto& q : pr) makespan = std::max(makespan, q.t);
        return makespan;
    }

    template <class WakeS, class WakeR>
    Step step(Proc& p, std::vector<Chan>& ch, uint64_t latency, WakeS& wake_senders, WakeR& wake_receivers) {
        const bool resumed = p.resumed;
        p.resumed = false;
        while (!p.stack.empty()) {
            Frame& f = p.stack.back();
            const Node& n = *f.node;
            switch (n.kind) {
                case Node::Kind::SlotSet:
                case Node::Kind::SlotLoad:
                    if (csp) csp->fail("slot operations in a process");
                    node(n, 0);
                    p.stack.pop_back();
                    break;
                case Node::Kind::Task:
                    enqueue(n);
                    p.t += P.impls[n.kernel_index].cycles;
                    p.stack.pop_back();
                    break;
                case Node::Kind::ParallelFor:
                case Node::Kind::ForEach: {
                    if (f.state == 0) {
                        if (n.axis.kind == Axis::Kind::Dense) f.ub = n.axis.size;
                        else if (n.axis.kind == Axis::Kind::DenseDyn) f.ub = axis_size(n.var);
                        else throw Error(PTOWSP_ERR_UNSUPPORTED, "CSPT codegen: unsupported axis kind in loop");
                        env.push_back({&n.var, 0});
                        f.state = 1;
                    }
                    if (f.i < f.ub) {
                        env.back().second = f.i++;
                        p.stack.push_back(Frame{n.body.get()});
                    } else {
                        env.pop_back();
                        p.stack.pop_back();
                    }
                    break;
                }
                case Node::Kind::Combine:
                case Node::Kind::Sequential:
                    if (f.i < static_cast<int64_t>(n.children.size())) p.stack.push_back(Frame{n.children[f.i++].get()});
                    else p.stack.pop_back();
                    break;
                case Node::Kind::Cond: {
                    const Node* br = eval(*n.pred, nullptr).v ? n.then_n.get() : n.else_n.get();
                    p.stack.back() = Frame{br};
                    break;
                }
                case Node::Kind::Send: {
                    Chan& c = ch[n.channel];
                    if (f.state == 0) {  // run the task, then offer its first axis arg
                        const std::vector<uint64_t> args = enqueue(*n.body);
                        p.t += P.impls[n.body->kernel_index].cycles;
                        p.token = n.body->axis_args.empty() ? 0 : args[0];
                        f.state = 1;
                    }
                    if (c.cap > 0) {
                        if (f.state == 2 && resumed && c.last_pop > p.t) p.t = c.last_pop;  // waited for room
                        if (c.closed) {
                            p.stack.pop_back();
                            return Step::Yield;
                        }
                        if (static_cast<int64_t>(c.buf.size()) >= c.cap) {
                            f.state = 2;
                            p.blocked = true;
                            p.wait_send = n.channel;
                            p.wait_recv = -1;
                            return Step::Blocked;
                        }
                        c.buf.push_back({p.token, p.t});
                        if (csp) csp_channel(n.channel, true);
                        wake_receivers(n.channel);
                        p.stack.pop_back();
                        return Step::Yield;
                    }
                    // rendezvous: wait for a waiting receiver, hand the token over, wait until it is taken
                    if (f.state == 1) {
                        if (c.closed) {
                            p.stack.pop_back();
                            return Step::Yield;
                        }
                        if (!c.receiver_waiting) {
                            p.blocked = true;
                            p.wait_send = n.channel;
                            p.wait_recv = -1;
                            return Step::Blocked;
                        }
                        c.rdv = {p.token, p.t};
                        c.has_rdv = true;
                        if (csp) csp_channel(n.channel, true);
                        wake_receivers(n.channel);
                        f.state = 3;
                    }
                    if (!c.closed && c.has_rdv) {
                        p.blocked = true;
                        p.wait_send = n.channel;
                        p.wait_recv = -1;
                        return Step::Blocked;
                    }
                    if (c.last_pop > p.t) p.t = c.last_pop;
                    p.stack.pop_back();
                    return Step::Yield;
                }
                case Node::Kind::Consume: {
                    Chan& c = ch[n.channel];
                    if (f.state == 1) {  // body done: unbind the token, receive the next one
                        env.pop_back();
                        f.state = 0;
                    }
                    bool got = false;
                    uint64_t tok = 0, ts = 0;
                    if (c.cap > 0) {
                        if (!c.buf.empty()) {
                            tok = c.buf.front().first;
                            ts = c.buf.front().second;
                            c.buf.pop_front();
                            got = true;
                        } else if (!c.closed) {
                            p.blocked = true;
                            p.wait_recv = n.channel;
                            p.wait_send = -1;
                            return Step::Blocked;
                        }
                    } else {
                        c.receiver_waiting = true;
                        wake_senders(n.channel);
                        if (!c.closed && !c.has_rdv) {
                            p.blocked = true;
                            p.wait_recv = n.channel;
                            p.wait_send = -1;
                            return Step::Blocked;
                        }
                        c.receiver_waiting = false;
                        if (c.has_rdv) {
                            tok = c.rdv.first;
                            ts = c.rdv.second;
                            c.has_rdv = false;
                            got = true;
                        }
                    }
                    if (!got) {  // closed and drained
                        p.stack.pop_back();
                        break;
                    }
                    if (csp) csp_channel(n.channel, false);
                    const uint64_t deliver = ts + latency;
                    if (deliver > p.t) p.t = deliver;
                    c.last_pop = p.t;
                    wake_senders(n.channel);
                    env.push_back({&n.var, static_cast<int64_t>(tok)});
                    f.state = 1;
                    p.stack.push_back(Frame{n.body.get()});
                    return Step::Yield;
                }
                default:
                    throw Error(PTOWSP_ERR_UNSUPPORTED, "CSPT codegen: unsupported node kind in process body");
            }
        }
        return Step::Done;
    }
};

}  // namespace

// ---------------------------------------------------------------------------

Batch::~Batch() {
    if (fast_rec_dev) cudaFree(fast_rec_dev);
    if (unit_rec_dev) cudaFree(unit_rec_dev);
    if (ep_mm_rec_dev) cudaFree(ep_mm_rec_dev);
    if (ep_rec_dev) cudaFree(ep_rec_dev);
    if (ep_unit_rec_dev) cudaFree(ep_unit_rec_dev);
    if (st_rec_dev) cudaFree(st_rec_dev);
    if (sel_dev) cudaFree(sel_dev);
    if (sel_tree_dev) cudaFree(sel_tree_dev);
}

CspDevice::~CspDevice() {
    for (void* q : {static_cast<void*>(ops_dev), static_cast<void*>(first_dev), static_cast<void*>(rec_dev),
                    static_cast<void*>(caps_dev), static_cast<void*>(tb_dev), static_cast<void*>(prog_dev),
                    static_cast<void*>(counts_dev)})
        if (q) cudaFree(q);
}

LaunchProgram::~LaunchProgram() {
    if (rec_dev) cudaFree(rec_dev);
    if (expand) {
        if (expand->base_delta_dev) cudaFree(expand->base_delta_dev);
        if (expand->vars_dev) cudaFree(expand->vars_dev);
    }
}

void set_error(const std::string& msg) { g_err = msg; }
const char* last_error() { return g_err.c_str(); }

Program::~Program() {
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cached.reset();
    for (auto& ki : impls)
        if (ki.tp_dev) cudaFree(ki.tp_dev);
    for (char* b : dev_bufs)
        if (b) cudaFree(b);
    if (scratch) cudaFree(scratch);
    if (err_dev) cudaFree(err_dev);
    if (ev0) cudaEventDestroy(ev0);
    if (ev1) cudaEventDestroy(ev1);
    for (auto e : pipe_events) cudaEventDestroy(e);
    for (auto& ke : kev_pending) {
        cudaEventDestroy(ke.start);
        cudaEventDestroy(ke.end);
    }
    for (auto e : kev_free) cudaEventDestroy(e);
    if (h2d_stream) cudaStreamDestroy(h2d_stream);
    if (d2h_stream) cudaStreamDestroy(d2h_stream);
    if (own_stream) cudaStreamDestroy(own_stream);
    if (prev >= 0) cudaSetDevice(prev);
}

namespace {

void ensure_device_state(Program& p) {
    if (!p.own_stream) {
        PW_CUDA(cudaStreamCreateWithFlags(&p.own_stream, cudaStreamNonBlocking));
        if (!p.stream_set) p.stream = p.own_stream;
        PW_CUDA(cudaEventCreate(&p.ev0));
        PW_CUDA(cudaEventCreate(&p.ev1));
        PW_CUDA(cudaMalloc(&p.err_dev, sizeof(int)));
        PW_CUDA(cudaMemset(p.err_dev, 0, sizeof(int)));
    }
    for (auto& ki : p.impls) {
        if (ki.tp_ok && !ki.tp_dev) {
            PW_CUDA(cudaMalloc(&ki.tp_dev, sizeof(dev::TileProgram)));
            PW_CUDA(cudaMemcpy(ki.tp_dev, &ki.tp, sizeof(dev::TileProgram), cudaMemcpyHostToDevice));
        }
    }
}

void* ensure_scratch(Program& p, size_t bytes) {
    if (bytes == 0) return nullptr;
    if (p.scratch_cap < bytes) {
        if (p.scratch) PW_CUDA(cudaFree(p.scratch));
        p.scratch = nullptr;
        p.scratch_cap = 0;
        PW_CUDA(cudaMalloc(&p.scratch, bytes));
        p.scratch_cap = bytes;
    }
    return p.scratch;
}

// Launch one batch.  `node` is the task node whose tensor bindings the batch uses.
// The record layout and tensor params of kernel `kernel`'s tasks under task node `node` with the current tensor
// bindings; rows_ok becomes false when a param's rows are not 16-byte aligned with unit column stride.
void fill_task_params(Program& P, int kernel, const Node& node, std::vector<TensorBinding>& T, dev::TaskBatch& tb,
                      bool& rows_ok) {
    const KernelDef& kd = P.plan.kernels[kernel];
    tb.stride = kd.num_tensor_params + static_cast<int>(node.axis_args.size()) + kd.num_scalar_params;
    tb.nparams = kd.num_tensor_params;
    tb.naxis = static_cast<int>(node.axis_args.size());
    tb.nscalar = kd.num_scalar_params;
    tb.err = P.err_dev;
    if (kd.num_tensor_params > dev::kMaxParams) throw Error(PTOWSP_ERR_LIMIT, "kernel has more than 8 tile params");
    for (const auto& kp : kd.params) {
        if (kp.tensor_index < 0) continue;
        const TensorArg& ta = node.tensor_args[node.param_to_arg[kp.tensor_index]];
        const TensorBinding& b = T[ta.tensor];
        dev::ParamDesc& pd = tb.p[kp.tensor_index];
        pd.base = b.dev;
        if (ta.view_rank >= 2) {
            pd.s3 = b.strides[ta.base_rank - ta.view_rank];
            pd.s4 = b.strides[ta.base_rank - ta.view_rank + 1];
        } else if (ta.view_rank == 1) {
            pd.s3 = 0;
            pd.s4 = b.strides[ta.base_rank - 1];
        } else {
            pd.s3 = 0;
            pd.s4 = 1;
        }
        pd.numel_span = b.span;
        pd.rows = kp.v.rows;
        pd.cols = kp.v.cols;
        pd.type = ptype(kp.v.dtype);
        pd.elem_bytes = dtype_bytes(kp.v.dtype);
        if (pd.s4 != 1 || (pd.s3 & 3) != 0 || (reinterpret_cast<uintptr_t>(pd.base) & 15) != 0) rows_ok = false;
    }
}

void launch_batch_body(Program& P, Batch& B, const Node& node, std::vector<TensorBinding>& T, const int64_t* rec_dev,
                       uint64_t& launches) {
    const KernelDef& kd = P.plan.kernels[B.kernel];
    KernelImpl& ki = P.impls[B.kernel];
    dev::TaskBatch tb{};
    bool rows_ok = B.aligned_rows;
    fill_task_params(P, B.kernel, node, T, tb, rows_ok);
    tb.rec = rec_dev + B.dev_off;
    tb.ntasks = B.ntasks;
    tb.stride = B.stride;
    const int workers = P.plan.schedule.window_tasks > 0 ? static_cast<int>(std::min<int64_t>(P.plan.schedule.window_tasks, 1 << 30)) : 0;
    cudaError_t e = cudaSuccess;
    ImplKind kind = ki.kind;
    if (B.sel) {
        // the scalars of every task come from the leaf its tensor element picks: write them into the records first
        if (!B.sel_dev) {
            const DevSelect& ds = *B.sel;
            std::vector<int> tree;
            static const char* cmps[] = {"<", "<=", ">", ">=", "==", "!="};
            for (size_t c = 0; c < ds.cmp.size(); ++c) {
                int code = 5;
                for (int k = 0; k < 6; ++k)
                    if (ds.cmp[c] == cmps[k]) code = k;
                tree.insert(tree.end(), {code, ds.slot_left[c], ds.then_c[c], ds.else_c[c]});
            }
            PW_CUDA(cudaMalloc(&B.sel_dev, B.sel_rows.size() * sizeof(uint64_t)));
            PW_CUDA(cudaMemcpy(B.sel_dev, B.sel_rows.data(), B.sel_rows.size() * sizeof(uint64_t), cudaMemcpyHostToDevice));
            PW_CUDA(cudaMalloc(&B.sel_tree_dev, tree.size() * sizeof(int)));
            PW_CUDA(cudaMemcpy(B.sel_tree_dev, tree.data(), tree.size() * sizeof(int), cudaMemcpyHostToDevice));
        }
        const TensorBinding& sb = T[B.sel_tensor];
        const int nscal = static_cast<int>(B.sel->leaves[0]->scalar_args.size());
        e = dev::launch_select_scalars(const_cast<int64_t*>(rec_dev) + B.dev_off, B.stride,
                                       kd.num_tensor_params + static_cast<int>(node.axis_args.size()), B.sel_dev,
                                       static_cast<int64_t>(B.sel_rows.size() / B.sel_row_words), B.sel_row_words,
                                       B.sel_tree_dev, static_cast<int>(B.sel->cmp.size()), nscal, sb.dev,
                                       static_cast<int>(P.plan.tensors[B.sel_tensor].dtype), sb.span, P.err_dev,
                                       P.stream);
        if (e != cudaSuccess) throw Error(PTOWSP_ERR_CUDA, std::string("device-selected scalars: ") + cudaGetErrorString(e));
        launches++;
    }
    if ((kind == ImplKind::RmsNorm || kind == ImplKind::Softmax)) {
        const int c = kd.params[0].v.cols;
        if (!rows_ok || !dev::row_width_supported(c)) kind = ImplKind::TileProgram;
    }
    if ((kind == ImplKind::Matmul || kind == ImplKind::MatmulAcc) && !ki.tp_ok && B.fast_ok == 0)
        throw Error(PTOWSP_ERR_UNSUPPORTED, "kernel '" + kd.name + "': operands do not meet the tcgen05 layout "
                                            "conditions and the tiles exceed the generic tile program");
    if (kind == ImplKind::Matmul || kind == ImplKind::MatmulAcc) {
        // tcgen05 path: shape/stride/alignment conditions, then every task's TMA coordinates
        if (B.fast_ok < 0) {
            bool ok = dev::matmul_tiles_supported(tb) && !B.rec.empty();
            const dev::ParamDesc &A = tb.p[0], &Bm = tb.p[1], &Cm = tb.p[2];
            const int64_t K = A.cols, N = Bm.cols;
            const int64_t a_rows = ok ? (A.numel_span + A.s3 - 1) / A.s3 : 0;
            const int64_t b_rows = ok ? (Bm.numel_span + Bm.s3 - 1) / Bm.s3 : 0;
            for (int64_t t = 0; ok && t < B.ntasks; ++t) {
                const int64_t* r = &B.rec[t * B.stride];
                const int64_t oa = r[0], ob = r[1], oc = r[2];
                ok = oa >= 0 && ob >= 0 && oc >= 0 && oa % 8 == 0 && ob % 8 == 0 && oc % 4 == 0 &&
                     (oa % A.s3) + K <= A.s3 && (oa / A.s3) + 128 <= a_rows && (ob % Bm.s3) + N <= Bm.s3 &&
                     (ob / Bm.s3) + K <= b_rows && oc + 127 * Cm.s3 + N <= Cm.numel_span;
            }
            B.fast_ok = ok ? 1 : 0;
            B.fast_n = static_cast<int>(N);
            B.fast_ntasks = B.ntasks;
            // pair tasks (t, t+1) that share A and cover adjacent N tiles of B and C
            if (ok && N == 128 && B.ntasks % 2 == 0) {
                bool pair = true;
                for (int64_t t = 0; pair && t < B.ntasks; t += 2) {
                    const int64_t* r0 = &B.rec[t * B.stride];
                    const int64_t* r1 = &B.rec[(t + 1) * B.stride];
                    pair = r1[0] == r0[0] && r1[1] == r0[1] + N && r1[2] == r0[2] + N &&
                           (r0[1] % Bm.s3) + 2 * N <= Bm.s3 && r0[2] + 127 * Cm.s3 + 2 * N <= Cm.numel_span;
                }
                if (pair) {
                    std::vector<int64_t> m(static_cast<size_t>(B.ntasks / 2) * 3);
                    for (int64_t t = 0; t < B.ntasks; t += 2)
                        for (int j = 0; j < 3; ++j) m[(t / 2) * 3 + j] = B.rec[t * B.stride + j];
                    PW_CUDA(cudaMalloc(&B.fast_rec_dev, m.size() * sizeof(int64_t)));
                    PW_CUDA(cudaMemcpy(B.fast_rec_dev, m.data(), m.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
                    B.fast_ntasks = B.ntasks / 2;
                    B.fast_n = 2 * static_cast<int>(N);
                    B.units_ok = -1;
                }
            }
            // CTA pairs: each (merged) task with the task 128 rows below it in A and C that shares its B tile
            if (ok && B.units_ok < 0) {
                std::vector<int64_t> r3;  // [oa, ob, oc] per task as launched
                if (B.fast_rec_dev) {
                    r3.resize(static_cast<size_t>(B.fast_ntasks) * 3);
                    for (int64_t t = 0; t < B.ntasks; t += 2)
                        for (int j = 0; j < 3; ++j) r3[(t / 2) * 3 + j] = B.rec[t * B.stride + j];
                } else {
                    r3.resize(static_cast<size_t>(B.ntasks) * 3);
                    for (int64_t t = 0; t < B.ntasks; ++t)
                        for (int j = 0; j < 3; ++j) r3[t * 3 + j] = B.rec[t * B.stride + j];
                }
                const int64_t n = static_cast<int64_t>(r3.size() / 3);
                std::unordered_map<uint64_t, int64_t> at;  // (oa, ob) -> task
                at.reserve(static_cast<size_t>(n) * 2);
                constexpr int64_t BM_ROWS = 128;  // rows of a task's A / C tile
                auto key = [](int64_t oa, int64_t ob) {  // splitmix64 finaliser of the pair
                    uint64_t z = static_cast<uint64_t>(oa) * 0x9e3779b97f4a7c15ull ^ static_cast<uint64_t>(ob);
                    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
                    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
                    return z ^ (z >> 31);
                };
                bool fine = n % 2 == 0 && (B.fast_n == 128 || B.fast_n == 256);
                for (int64_t t = 0; fine && t < n; ++t) fine = at.emplace(key(r3[t * 3], r3[t * 3 + 1]), t).second;
                std::vector<char> used(static_cast<size_t>(n), 0);
                std::vector<int64_t> units;
                units.reserve(static_cast<size_t>(n) * 3);
                for (int64_t t = 0; fine && t < n; ++t) {
                    if (used[t]) continue;
                    const int64_t oa = r3[t * 3], ob = r3[t * 3 + 1], oc = r3[t * 3 + 2];
                    auto it = at.find(key(oa + BM_ROWS * A.s3, ob));
                    fine = it != at.end() && !used[it->second] && r3[it->second * 3] == oa + BM_ROWS * A.s3 &&
                           r3[it->second * 3 + 1] == ob && r3[it->second * 3 + 2] == oc + BM_ROWS * Cm.s3;
                    if (!fine) break;
                    used[t] = used[it->second] = 1;
                    for (int j = 0; j < 3; ++j) units.push_back(r3[t * 3 + j]);
                    for (int j = 0; j < 3; ++j) units.push_back(r3[it->second * 3 + j]);
                }
                B.units_ok = fine ? 1 : 0;
                if (fine) {
                    PW_CUDA(cudaMalloc(&B.unit_rec_dev, units.size() * sizeof(int64_t)));
                    PW_CUDA(cudaMemcpy(B.unit_rec_dev, units.data(), units.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
                    B.nunits = static_cast<int64_t>(units.size() / 6);
                }
            }
        }
        if (!B.fast_ok) kind = ImplKind::TileProgram;
        if (B.fast_ok && B.fast_rec_dev) {
            tb.rec = B.fast_rec_dev;
            tb.ntasks = B.fast_ntasks;
            tb.stride = 3;
            tb.p[1].cols = B.fast_n;
            tb.p[2].cols = B.fast_n;
        }
    }
    dev::ParamDesc ep_tile{};  // MatmulEpilogue: the scratch tile between the two launches
    if (kind == ImplKind::MatmulEpilogue) {
        const int np = kd.num_tensor_params;
        const int64_t tile = int64_t(128) * ki.ep_n;
        ep_tile.base = static_cast<char*>(ensure_scratch(P, static_cast<size_t>(B.ntasks) * tile * sizeof(float)));
        ep_tile.s3 = ki.ep_n;
        ep_tile.s4 = 1;
        ep_tile.numel_span = B.ntasks * tile;
        ep_tile.rows = 128;
        ep_tile.cols = ki.ep_n;
        ep_tile.type = dev::PT_F32;
        ep_tile.elem_bytes = 4;
        if (B.ep_ok < 0) {
            // records of both stages, from the host records (read back once when a cached table dropped them)
            std::vector<int64_t> back;
            const int64_t* rec = B.rec.data();
            if (B.rec.empty()) {
                back.resize(static_cast<size_t>(B.ntasks) * B.stride);
                PW_CUDA(cudaMemcpyAsync(back.data(), rec_dev + B.dev_off, back.size() * sizeof(int64_t),
                                        cudaMemcpyDeviceToHost, P.stream));
                PW_CUDA(cudaStreamSynchronize(P.stream));
                rec = back.data();
            }
            dev::TaskBatch mtb{};
            mtb.p[0] = tb.p[ki.ep_a];
            mtb.p[1] = tb.p[ki.ep_b];
            mtb.p[2] = ep_tile;
            bool ok = dev::matmul_tiles_supported(mtb) && B.ntasks > 0;
            const dev::ParamDesc &A = mtb.p[0], &Bm = mtb.p[1];
            const int64_t K = ki.ep_k, N = ki.ep_n;
            const int64_t a_rows = ok ? (A.numel_span + A.s3 - 1) / A.s3 : 0;
            const int64_t b_rows = ok ? (Bm.numel_span + Bm.s3 - 1) / Bm.s3 : 0;
            std::vector<int64_t> mm(static_cast<size_t>(B.ntasks) * 3), er(static_cast<size_t>(B.ntasks) * (B.stride + 1));
            for (int64_t t = 0; ok && t < B.ntasks; ++t) {
                const int64_t* r = rec + t * B.stride;
                const int64_t oa = r[ki.ep_a], ob = r[ki.ep_b];
                ok = oa >= 0 && ob >= 0 && oa % 8 == 0 && ob % 8 == 0 && (oa % A.s3) + K <= A.s3 &&
                     (oa / A.s3) + 128 <= a_rows && (ob % Bm.s3) + N <= Bm.s3 && (ob / Bm.s3) + K <= b_rows;
                mm[t * 3] = oa;
                mm[t * 3 + 1] = ob;
                mm[t * 3 + 2] = t * tile;
                int64_t* o = &er[t * (B.stride + 1)];
                for (int j = 0; j < np; ++j) o[j] = r[j];
                o[np] = t * tile;
                for (int j = np; j < B.stride; ++j) o[j + 1] = r[j];
            }
            B.ep_ok = ok ? 1 : 0;
            if (ok && (N == 128 || N == 256) && B.ntasks % 2 == 0) {
                // CTA pairs for the matmul stage: each task with the task 128 rows below it in A that reads the
                // same B tile (each CTA stores its own scratch tile)
                std::unordered_map<uint64_t, int64_t> at;
                at.reserve(static_cast<size_t>(B.ntasks) * 2);
                auto key = [](int64_t oa, int64_t ob) {  // splitmix64 finaliser of the pair
                    uint64_t z = static_cast<uint64_t>(oa) * 0x9e3779b97f4a7c15ull ^ static_cast<uint64_t>(ob);
                    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
                    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
                    return z ^ (z >> 31);
                };
                bool fine = true;
                for (int64_t t = 0; fine && t < B.ntasks; ++t) fine = at.emplace(key(mm[t * 3], mm[t * 3 + 1]), t).second;
                std::vector<char> used(static_cast<size_t>(B.ntasks), 0);
                std::vector<int64_t> units;
                units.reserve(static_cast<size_t>(B.ntasks) * 3);
                for (int64_t t = 0; fine && t < B.ntasks; ++t) {
                    if (used[t]) continue;
                    auto it = at.find(key(mm[t * 3] + 128 * A.s3, mm[t * 3 + 1]));
                    fine = it != at.end() && !used[it->second] && mm[it->second * 3] == mm[t * 3] + 128 * A.s3 &&
                           mm[it->second * 3 + 1] == mm[t * 3 + 1];
                    if (!fine) break;
                    used[t] = used[it->second] = 1;
                    for (int j = 0; j < 3; ++j) units.push_back(mm[t * 3 + j]);
                    for (int j = 0; j < 3; ++j) units.push_back(mm[it->second * 3 + j]);
                }
                if (fine) {
                    PW_CUDA(cudaMalloc(&B.ep_unit_rec_dev, units.size() * sizeof(int64_t)));
                    PW_CUDA(cudaMemcpy(B.ep_unit_rec_dev, units.data(), units.size() * sizeof(int64_t),
                                       cudaMemcpyHostToDevice));
                    B.ep_nunits = static_cast<int64_t>(units.size() / 6);
                }
            }
            if (ok) {
                PW_CUDA(cudaMalloc(&B.ep_mm_rec_dev, mm.size() * sizeof(int64_t)));
                PW_CUDA(cudaMemcpy(B.ep_mm_rec_dev, mm.data(), mm.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
                PW_CUDA(cudaMalloc(&B.ep_rec_dev, er.size() * sizeof(int64_t)));
                PW_CUDA(cudaMemcpy(B.ep_rec_dev, er.data(), er.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
            }
        }
        if (ki.ep_jit_state == 2) {
            const std::string name = "ptowsp_ep_k" + std::to_string(B.kernel);
            std::string note;
            if (jit::load_cubin(ki.ep_cubin, name, &ki.ep_fn, &note)) {
                ki.ep_jit_state = 1;
                if (!jit::load_cubin(ki.ep_cubin, name + "_v", &ki.ep_fn_vec, &note)) ki.ep_fn_vec = nullptr;
            } else {
                ki.ep_jit_state = -1;
                ki.jit_note = note;
            }
        }
        if (B.ep_ok != 1 || ki.ep_jit_state != 1) kind = ImplKind::TileProgram;  // the generic tile program
    }
    // Staged: f32 scratch tiles, one per task and crossing value, and the stage records (built once per batch)
    const int st_np = kd.num_tensor_params;
    const int st_S = static_cast<int>(ki.scratch_tiles.size());
    std::vector<int64_t> st_base(static_cast<size_t>(st_S) + 1, 0);
    char* st_scr = nullptr;
    auto st_tile = [&](int j) { return int64_t(ki.scratch_tiles[j].first) * ki.scratch_tiles[j].second; };
    auto st_desc = [&](int j) {
        dev::ParamDesc d{};
        d.base = st_scr;
        d.s3 = ki.scratch_tiles[j].second;
        d.s4 = 1;
        d.numel_span = st_base[st_S];
        d.rows = ki.scratch_tiles[j].first;
        d.cols = ki.scratch_tiles[j].second;
        d.type = dev::PT_F32;
        d.elem_bytes = 4;
        return d;
    };
    const int st_stride = B.stride + st_S;
    auto st_mm_records = [&](int64_t ntasks) {  // matmul-stage records: n / tn per task for tcgen05 candidates
        int64_t n = 0;
        for (const auto& st : ki.stages)
            if (st.mm) n += ntasks * (st.tc ? st.n / st.tn : 1);
        return n;
    };
    bool st_rows_ok = rows_ok;
    if (kind == ImplKind::Attention && !P.opt_fused_attention) kind = ImplKind::Staged;
    if (kind == ImplKind::Attention) {
        // the fused kernel takes the batch when every task's views meet its layout conditions (checked once per
        // batch, from the host records or, when a cached task table dropped them, a copy read back)
        if (B.at_ok < 0) {
            bool ok = dev::attention_tiles_supported(tb, ki.at_q, ki.at_kt, ki.at_v, ki.at_o, ki.at_L);
            std::vector<int64_t> back;
            const int64_t* rec = B.rec.data();
            if (ok && B.rec.empty() && B.ntasks > 0) {
                back.resize(static_cast<size_t>(B.ntasks) * B.stride);
                PW_CUDA(cudaMemcpyAsync(back.data(), rec_dev + B.dev_off, back.size() * sizeof(int64_t),
                                        cudaMemcpyDeviceToHost, P.stream));
                PW_CUDA(cudaStreamSynchronize(P.stream));
                rec = back.data();
            }
            for (int64_t t = 0; ok && t < B.ntasks; ++t)
                ok = dev::attention_task_ok(tb, ki.at_q, ki.at_kt, ki.at_v, ki.at_o, ki.at_L, rec + t * B.stride);
            B.at_ok = ok ? 1 : 0;
        }
        if (!B.at_ok) kind = ImplKind::Staged;
    }
    // the stages run over groups of st_group tasks, so that the scratch stays within the stage_scratch_mb budget
    // (2 GiB by default) whatever the batch; the group is fixed when the batch's records are built
    int64_t st_group = B.ntasks;
    if (kind == ImplKind::Staged) {
        int64_t per_task = 0;
        for (int j = 0; j < st_S; ++j) per_task += st_tile(j);
        const int64_t budget = (P.opt_stage_scratch_mb << 20) / static_cast<int64_t>(sizeof(float));
        st_group = std::max<int64_t>(1, std::min<int64_t>(B.ntasks, budget / std::max<int64_t>(per_task, 1)));
        if (B.st_ok > 0) st_group = B.st_group;
        B.st_group = st_group;
        for (int j = 0; j < st_S; ++j) {
            st_base[j + 1] = st_base[j] + st_group * st_tile(j);
            if (ki.scratch_tiles[j].second % 4) st_rows_ok = false;
        }
        st_scr = static_cast<char*>(ensure_scratch(P, static_cast<size_t>(st_base[st_S]) * sizeof(float)));
        if (B.st_ok < 0) {
            // records of every stage, from the host records (read back once when a cached table dropped them)
            std::vector<int64_t> back;
            const int64_t* rec = B.rec.data();
            if (B.rec.empty()) {
                back.resize(static_cast<size_t>(B.ntasks) * B.stride);
                PW_CUDA(cudaMemcpyAsync(back.data(), rec_dev + B.dev_off, back.size() * sizeof(int64_t),
                                        cudaMemcpyDeviceToHost, P.stream));
                PW_CUDA(cudaStreamSynchronize(P.stream));
                rec = back.data();
            }
            std::vector<int64_t> all(static_cast<size_t>(B.ntasks) * st_stride + 3 * st_mm_records(B.ntasks));
            for (int64_t t = 0; t < B.ntasks; ++t) {
                const int64_t* r = rec + t * B.stride;
                int64_t* o = &all[t * st_stride];
                for (int j = 0; j < st_np; ++j) o[j] = r[j];
                for (int j = 0; j < st_S; ++j) o[st_np + j] = st_base[j] + (t % st_group) * st_tile(j);
                for (int j = st_np; j < B.stride; ++j) o[j + st_S] = r[j];
            }
            B.st_tc_mask = 0;
            int q = 0;
            size_t mo = static_cast<size_t>(B.ntasks) * st_stride;  // this matmul stage's records
            for (const auto& st : ki.stages) {
                if (!st.mm) continue;
                int64_t* m = &all[mo];
                auto off = [&](int src, int64_t t, const int64_t* r) {
                    return src >= 0 ? r[src] : st_base[~src] + (t % st_group) * st_tile(~src);
                };
                bool ok = st.tc;
                if (ok) {
                    // tcgen05 tile kernel: each task's n columns as n / tn tiles [oa, ob + j tn, oc + j tn], under
                    // the kernel's layout conditions for every tile
                    const int ns = st.n / st.tn;
                    dev::TaskBatch mtb{};
                    mtb.p[0] = tb.p[st.a];
                    mtb.p[1] = tb.p[st.b];
                    mtb.p[1].cols = st.tn;
                    mtb.p[2] = st_desc(st.c);
                    mtb.p[2].cols = st.tn;
                    ok = dev::matmul_tiles_supported(mtb) && mtb.p[1].s4 == 1;
                    const dev::ParamDesc &A = mtb.p[0], &Bm = mtb.p[1];
                    const int64_t a_rows = ok ? (A.numel_span + A.s3 - 1) / A.s3 : 0;
                    const int64_t b_rows = ok ? (Bm.numel_span + Bm.s3 - 1) / Bm.s3 : 0;
                    for (int64_t t = 0; ok && t < B.ntasks; ++t) {
                        const int64_t* r = rec + t * B.stride;
                        const int64_t oa = off(st.a, t, r), ob = off(st.b, t, r);
                        const int64_t oc = st_base[st.c] + (t % st_group) * st_tile(st.c);
                        ok = oa >= 0 && ob >= 0 && oa % 8 == 0 && ob % 8 == 0 && (oa % A.s3) + st.k <= A.s3 &&
                             (oa / A.s3) + 128 <= a_rows && (ob % Bm.s3) + st.n <= Bm.s3 && (ob / Bm.s3) + st.k <= b_rows;
                        for (int j = 0; ok && j < ns; ++j) {
                            int64_t* x = &m[(t * ns + j) * 3];
                            x[0] = oa;
                            x[1] = ob + static_cast<int64_t>(j) * st.tn;
                            x[2] = oc + static_cast<int64_t>(j) * st.tn;
                        }
                    }
                    if (ok) B.st_tc_mask |= 1u << q;
                }
                if (!ok) {  // CUDA-core kernel: one record per task
                    for (int64_t t = 0; t < B.ntasks; ++t) {
                        const int64_t* r = rec + t * B.stride;
                        m[t * 3] = off(st.a, t, r);
                        m[t * 3 + 1] = off(st.b, t, r);
                        m[t * 3 + 2] = st_base[st.c] + (t % st_group) * st_tile(st.c);
                    }
                }
                mo += 3 * static_cast<size_t>(B.ntasks) * (st.tc ? st.n / st.tn : 1);
                ++q;
            }
            PW_CUDA(cudaMalloc(&B.st_rec_dev, all.size() * sizeof(int64_t)));
            PW_CUDA(cudaMemcpy(B.st_rec_dev, all.data(), all.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
            B.st_ok = 1;
        }
        for (size_t si = 0; si < ki.stages.size(); ++si) {
            Stage& st = ki.stages[si];
            if (st.mm || st.jit_state != 2) continue;
            const std::string name = "ptowsp_st_k" + std::to_string(B.kernel) + "_" + std::to_string(si);
            std::string note;
            if (!jit::load_cubin(st.cubin, name, &st.fn, &note))
                throw Error(PTOWSP_ERR_CUDA, "kernel '" + kd.name + "': stage " + std::to_string(si) + ": " + note);
            st.jit_state = 1;
            if (!jit::load_cubin(st.cubin, name + "_v", &st.fn_vec, &note)) st.fn_vec = nullptr;
        }
    }
    switch (kind) {
        case ImplKind::Attention:
            e = dev::launch_attention(tb, ki.at_q, ki.at_kt, ki.at_v, ki.at_o, ki.at_L, ki.at_scale_mode,
                                      kd.num_tensor_params + tb.naxis + std::max(ki.at_scale_index, 0),
                                      ki.at_scale_const, P.stream);
            break;
        case ImplKind::Staged: {
            bool first = true;
            for (int64_t t0 = 0; t0 < B.ntasks && e == cudaSuccess; t0 += st_group) {
                const int64_t n = std::min<int64_t>(st_group, B.ntasks - t0);
                int q = 0;
                size_t mo = static_cast<size_t>(B.ntasks) * st_stride;
                for (size_t si = 0; si < ki.stages.size(); ++si) {
                    const Stage& st = ki.stages[si];
                    if (!first) launches++;  // every launch but the last is counted here, the last below
                    first = false;
                    if (st.mm) {
                        const bool tc = (B.st_tc_mask >> q) & 1u;
                        const int64_t split = tc ? st.n / st.tn : 1;
                        dev::TaskBatch mtb{};
                        mtb.p[0] = st.a >= 0 ? tb.p[st.a] : st_desc(~st.a);
                        mtb.p[1] = st.b >= 0 ? tb.p[st.b] : st_desc(~st.b);
                        mtb.p[2] = st_desc(st.c);
                        mtb.rec = B.st_rec_dev + mo + static_cast<size_t>(t0 * split) * 3;
                        mtb.ntasks = n * split;
                        mtb.stride = 3;
                        mtb.nparams = 3;
                        mtb.err = P.err_dev;
                        if (tc) {
                            mtb.p[1].cols = st.tn;
                            mtb.p[2].cols = st.tn;
                            e = dev::launch_matmul_tiles(mtb, 0, workers, P.stream);
                        } else {
                            e = dev::launch_matmul_simt(mtb, st.m, st.n, st.k, workers, P.stream);
                        }
                        mo += 3 * static_cast<size_t>(B.ntasks) * (st.tc ? st.n / st.tn : 1);
                        ++q;
                    } else {
                        dev::TaskBatch etb = tb;
                        for (int j = 0; j < st_S; ++j) etb.p[st_np + j] = st_desc(j);
                        etb.nparams = st_np + st_S;
                        etb.stride = st_stride;
                        etb.rec = B.st_rec_dev + static_cast<size_t>(t0) * st_stride;
                        etb.ntasks = n;
                        e = jit::launch_row_kernel(st_rows_ok && st.fn_vec ? st.fn_vec : st.fn, etb, st.rows, workers,
                                                   P.stream);
                    }
                    if (e != cudaSuccess) break;
                }
            }
            break;
        }
        case ImplKind::MatmulEpilogue: {
            const int np = kd.num_tensor_params;
            dev::TaskBatch mtb{};
            mtb.p[0] = tb.p[ki.ep_a];
            mtb.p[1] = tb.p[ki.ep_b];
            mtb.p[2] = ep_tile;
            mtb.rec = B.ep_mm_rec_dev;
            mtb.ntasks = B.ntasks;
            mtb.stride = 3;
            mtb.nparams = 3;
            mtb.err = P.err_dev;
            cudaError_t pe = cudaSuccess;
            if (B.ep_unit_rec_dev && dev::launch_matmul_pairs(mtb, B.ep_unit_rec_dev, B.ep_nunits, 0, workers, P.stream, &pe))
                e = pe;
            else
                e = dev::launch_matmul_tiles(mtb, 0, workers, P.stream);
            if (e != cudaSuccess) break;
            launches++;
            dev::TaskBatch etb = tb;
            etb.p[np] = ep_tile;
            etb.nparams = np + 1;
            etb.stride = B.stride + 1;
            etb.rec = B.ep_rec_dev;
            e = jit::launch_row_kernel(rows_ok && ki.ep_fn_vec ? ki.ep_fn_vec : ki.ep_fn, etb, 128, workers, P.stream);
            break;
        }
        case ImplKind::RmsNorm: e = dev::launch_rmsnorm_rows(tb, workers, P.stream); break;
        case ImplKind::Softmax: e = dev::launch_softmax_rows(tb, workers, P.stream); break;
        case ImplKind::Matmul:
        case ImplKind::MatmulAcc: {
            const int acc = kind == ImplKind::MatmulAcc ? 1 : 0;
            cudaError_t pe = cudaSuccess;
            if (B.units_ok == 1 && dev::launch_matmul_pairs(tb, B.unit_rec_dev, B.nunits, acc, workers, P.stream, &pe)) {
                e = pe;
                break;
            }
            e = dev::launch_matmul_tiles(tb, acc, workers, P.stream);
            break;
        }
        case ImplKind::TileProgram:
            if (!ki.tp_ok) throw Error(PTOWSP_ERR_UNSUPPORTED, "kernel '" + kd.name + "': " + ki.tp_error);
            if (ki.jit_state == 0) jit_prepare(ki, kd, B.kernel);  // a fast-path kernel that fell back here
            if (ki.jit_state == 2) {
                const std::string name = "ptowsp_rows_k" + std::to_string(B.kernel);
                void* fn = nullptr;
                if (jit::load_cubin(ki.jit_cubin, name, &fn, &ki.jit_note)) {
                    ki.jit_fn = fn;
                    ki.jit_state = 1;
                    void* fv = nullptr;
                    std::string note;
                    if (jit::load_cubin(ki.jit_cubin, name + "_v", &fv, &note)) ki.jit_fn_vec = fv;  // absent: scalar only
                } else {
                    ki.jit_state = -1;
                }
            }
            if (ki.jit_state == 1)
                e = jit::launch_row_kernel(rows_ok && ki.jit_fn_vec ? ki.jit_fn_vec : ki.jit_fn, tb,
                                           jit::program_rows(ki.tp), workers, P.stream);
            else e = dev::launch_tile_program(tb, ki.tp_dev, ki.tp_smem, workers, P.stream);
            break;
        case ImplKind::PagedDecode: {
            const dev::ParamDesc &K = tb.p[1], &V = tb.p[2];
            const dev::ParamDesc& Q = tb.p[0];
            const bool aligned = K.s3 % 8 == 0 && K.s4 % 8 == 0 && V.s3 % 8 == 0 && V.s4 % 8 == 0 && Q.s3 % 8 == 0 &&
                                 Q.s4 == 1 &&
                                 ((reinterpret_cast<uintptr_t>(K.base) | reinterpret_cast<uintptr_t>(V.base) |
                                   reinterpret_cast<uintptr_t>(Q.base)) & 15) == 0;
            bool q_rows_ok = true;  // q rows are read 16 bytes at a time
            for (int64_t t = 0; t < B.ntasks && !B.rec.empty(); ++t) q_rows_ok = q_rows_ok && B.rec[t * B.stride] % 8 == 0;
            if (!aligned || !q_rows_ok)
                throw Error(PTOWSP_ERR_UNSUPPORTED, "paged_decode_gqa: q and KV cache rows must be 16-byte aligned");
            size_t sb = dev::paged_decode_scratch_bytes(tb, 16);
            void* s = ensure_scratch(P, sb);
            e = dev::launch_paged_decode(tb, 16, static_cast<int>(P.opt_decode_chunk), workers, s, sb, P.stream);
            break;
        }
        case ImplKind::IndexerScore: {
            if (B.fast_ok < 0) {
                bool ok = dev::indexer_score_supported(tb) && !B.rec.empty();
                for (int64_t t = 0; ok && t < B.ntasks; ++t) {
                    const int64_t* r = &B.rec[t * B.stride];
                    ok = r[0] % 128 == 0 && r[1] % 128 == 0 && r[2] % 4 == 0 && r[0] + 512 * 128 <= tb.p[0].numel_span &&
                         r[1] + tb.p[1].rows * 128 <= tb.p[1].numel_span;
                }
                B.fast_ok = ok ? 1 : 0;
            }
            if (!B.fast_ok)
                throw Error(PTOWSP_ERR_UNSUPPORTED, "lightning_indexer_score: q/k views must be dense [rows,128] f16 tiles");
            e = dev::launch_indexer_score(tb, workers, P.stream);
            break;
        }
        case ImplKind::TopK: {
            size_t sb = dev::topk_select_scratch_bytes(tb);
            void* s = ensure_scratch(P, sb);
            e = dev::launch_topk_select(tb, workers, s, sb, P.stream);
            break;
        }
        default: throw Error(PTOWSP_ERR_UNSUPPORTED, "no launcher");
    }
    if (e != cudaSuccess) throw Error(PTOWSP_ERR_CUDA, "launch of " + kd.name + ": " + cudaGetErrorString(e));
    launches++;
}


// Host-staged runs overlapped: a workload whose waves hold one batch each (a
// chain of kernels, e.g. scoring then top-k) is cut into chunks of consecutive
// tasks of every batch; chunk c's input ranges are copied in on a copy stream,
// its kernels (one per wave, in wave order) wait for them on the compute stream,
// and its output ranges go back on a second copy stream while later chunks
// compute.  Inputs are copied once (ranges already staged by an earlier chunk
// are skipped).  Only for chains whose written host tensors are fully
// overwritten, each by one wave and read only by later waves, where chunk c of
// a reader reads inside what chunk c of the writer wrote.
bool pipelinable_kind(const KernelImpl& ki, const Batch& B) {
    switch (ki.kind) {
        case ImplKind::RmsNorm:
        case ImplKind::Softmax:
        case ImplKind::TileProgram:
        case ImplKind::TopK: return true;
        // hand-written kernels whose per-batch layout check ran on an earlier launch: each chunk then runs the
        // plain form of the kernel on its own records (the one-CTA tile kernel for tcgen05 matmuls)
        case ImplKind::Matmul:
        case ImplKind::IndexerScore: return B.fast_ok == 1;
        default: return false;
    }
}

// Per chunk and tensor param, the [lo, hi) element range the chunk's tasks touch, and whether the tiles of a param
// cover each chunk's range exactly once (dense tiles, sorted offsets adjacent).
bool chunk_ranges(Program& P, LaunchProgram& L, const std::vector<TensorBinding>& T, Batch* B, int C, bool dry) {
    if (B->chunk_n == C) return true;
    if (dry && B->rec.empty()) return false;  // a host-only walk reads no device memory
    const KernelDef& kd = P.plan.kernels[B->kernel];
    const Node& node = *B->node;
    const int np = kd.num_tensor_params;
    std::vector<int64_t> ext(np, 1);
    std::vector<uint8_t> dense(np, 0);
    for (const auto& kp : kd.params) {
        if (kp.tensor_index < 0) continue;
        const TensorArg& ta = node.tensor_args[node.param_to_arg[kp.tensor_index]];
        const TensorBinding& tb = T[ta.tensor];
        int64_t s3 = 0, s4 = 1;
        if (ta.view_rank >= 2) {
            s3 = tb.strides[ta.base_rank - ta.view_rank];
            s4 = tb.strides[ta.base_rank - ta.view_rank + 1];
        } else if (ta.view_rank == 1) {
            s4 = tb.strides[ta.base_rank - 1];
        }
        ext[kp.tensor_index] = (kp.v.rows - 1) * s3 + (kp.v.cols - 1) * s4 + 1;
        dense[kp.tensor_index] = s4 == 1 && (kp.v.rows == 1 || s3 == kp.v.cols);
    }
    // the host records of a cached task table are dropped after its first run: read them back once
    std::vector<int64_t> back;
    const int64_t* rec = B->rec.data();
    if (B->rec.empty()) {
        back.resize(static_cast<size_t>(B->ntasks) * B->stride);
        PW_CUDA(cudaMemcpyAsync(back.data(), L.rec_dev + B->dev_off, back.size() * sizeof(int64_t),
                                cudaMemcpyDeviceToHost, P.stream));
        PW_CUDA(cudaStreamSynchronize(P.stream));
        rec = back.data();
    }
    B->chunk_ranges.assign(static_cast<size_t>(C) * np * 2, 0);
    B->chunk_exact.assign(static_cast<size_t>(np), 1);
    std::vector<int64_t> offs;
    for (int c = 0; c < C; ++c) {
        const int64_t t0 = B->ntasks * c / C, t1 = B->ntasks * (c + 1) / C;
        for (int ti = 0; ti < np; ++ti) {
            int64_t lo = INT64_MAX, hi = 0;
            offs.clear();
            for (int64_t t = t0; t < t1; ++t) {
                const int64_t off = rec[t * B->stride + ti];
                lo = std::min(lo, off);
                hi = std::max(hi, off + ext[ti]);
                offs.push_back(off);
            }
            B->chunk_ranges[(static_cast<size_t>(c) * np + ti) * 2] = lo;
            B->chunk_ranges[(static_cast<size_t>(c) * np + ti) * 2 + 1] = hi;
            bool exact = dense[ti] != 0;
            if (exact) {
                std::sort(offs.begin(), offs.end());
                for (size_t i = 1; exact && i < offs.size(); ++i) exact = offs[i] == offs[i - 1] + ext[ti];
                exact = exact && !offs.empty() && offs.front() == lo && offs.back() + ext[ti] == hi;
            }
            if (!exact) B->chunk_exact[ti] = 0;
        }
    }
    B->chunk_n = C;
    return true;
}

// Whether and how a host-staged run overlaps: the chain of batches, the wave producing each host tensor, the chunk
// count.  No CUDA call, except reading back the records of a cached task table once (never when `dry`).
struct PipePlan {
    std::vector<Batch*> chain;
    std::vector<int> producer;
    int C = 0;
};

bool plan_pipeline(Program& P, LaunchProgram& L, std::vector<TensorBinding>& T, bool dry, PipePlan& pp) {
    if (!P.cacheable || P.opt_chunks < 2 || L.waves.empty() || L.waves.size() > 8 || L.no_pipeline) return false;
    std::vector<Batch*>& chain = pp.chain;  // one batch per wave
    int64_t min_tasks = INT64_MAX;
    for (auto& w : L.waves) {
        if (w.batches.size() != 1) return false;
        Batch* B = &w.batches[0];
        if (B->ntasks < 2 || B->sel || !pipelinable_kind(P.impls[B->kernel], *B)) return false;
        chain.push_back(B);
        min_tasks = std::min(min_tasks, B->ntasks);
    }
    const int nw = static_cast<int>(chain.size());
    // host tensors: the wave writing each (one at most, fully overwritten, read only by later waves)
    struct Use {
        int wave, param;
    };
    pp.producer.assign(T.size(), -1);
    std::vector<int>& producer = pp.producer;
    std::vector<int> producer_param(T.size(), -1), first_read(T.size(), INT_MAX);
    std::vector<std::vector<Use>> reads(T.size());
    size_t host_bytes = 0;
    std::vector<uint8_t> counted(T.size(), 0);
    for (int w = 0; w < nw; ++w) {
        const Batch* B = chain[w];
        const KernelImpl& ki = P.impls[B->kernel];
        const Node& node = *B->node;
        const int np = P.plan.kernels[B->kernel].num_tensor_params;
        for (int ti = 0; ti < np; ++ti) {
            const uint32_t tid = node.tensor_args[node.param_to_arg[ti]].tensor;
            if (T[tid].on_device) continue;
            if (!counted[tid]) {
                counted[tid] = 1;
                host_bytes += T[tid].bytes;
            }
            if (ki.param_write[ti]) {
                if (producer[tid] >= 0 || first_read[tid] < w) return false;  // a second writer, or a write after a read
                if (L.full_write.empty() || !L.full_write[tid]) return false;
                producer[tid] = w;
                producer_param[tid] = ti;
            }
        }
        for (int ti = 0; ti < np; ++ti) {
            const uint32_t tid = node.tensor_args[node.param_to_arg[ti]].tensor;
            if (T[tid].on_device || !ki.param_read[ti]) continue;
            if (producer[tid] == w) return false;  // read and written by the same batch
            first_read[tid] = std::min(first_read[tid], w);
            reads[tid].push_back({w, ti});
        }
    }
    if (host_bytes < (size_t(64) << 20)) return false;  // small copies: not worth the extra streams
    // chunks of at least 4 MiB of host traffic: smaller copies do not reach the copy engines' rate
    const int64_t by_size = std::max<int64_t>(2, static_cast<int64_t>(host_bytes >> 22));
    const int C = static_cast<int>(std::min<int64_t>(std::min<int64_t>(P.opt_chunks, min_tasks), by_size));
    for (Batch* B : chain)
        if (!chunk_ranges(P, L, T, B, C, dry)) return false;
    auto range = [&](const Batch* B, int c, int ti, int k) {
        const int np = P.plan.kernels[B->kernel].num_tensor_params;
        return B->chunk_ranges[(static_cast<size_t>(c) * np + ti) * 2 + k];
    };
    for (const Batch* B : chain) {  // ranges must stay inside the tensors
        const Node& node = *B->node;
        const int np = P.plan.kernels[B->kernel].num_tensor_params;
        for (int ti = 0; ti < np; ++ti)
            for (int c = 0; c < C; ++c)
                if (range(B, c, ti, 0) < 0 ||
                    range(B, c, ti, 1) > T[node.tensor_args[node.param_to_arg[ti]].tensor].span)
                    return false;
    }
    // a tensor passed between waves: chunk c of each reader reads inside what chunk c of the writer wrote, and the
    // writer's chunks cover their ranges exactly (no element of a range left to a later chunk)
    for (size_t tid = 0; tid < T.size(); ++tid) {
        if (producer[tid] < 0 || reads[tid].empty()) continue;
        const Batch* Wb = chain[producer[tid]];
        const int wp = producer_param[tid];
        if (!Wb->chunk_exact[wp]) return false;
        for (const Use& u : reads[tid])
            for (int c = 0; c < C; ++c)
                if (range(chain[u.wave], c, u.param, 0) < range(Wb, c, wp, 0) ||
                    range(chain[u.wave], c, u.param, 1) > range(Wb, c, wp, 1))
                    return false;
    }
    pp.C = C;
    return true;
}

// launch_batch_body, bracketed by CUDA events on the launch stream when the "kernel_events" option is on
// (per-kernel device time, read by ptowsp_cuda_kernel_times).
void launch_batch(Program& P, Batch& B, const Node& node, std::vector<TensorBinding>& T, const int64_t* rec_dev,
                  uint64_t& launches) {
    if (!P.opt_kernel_events) {
        launch_batch_body(P, B, node, T, rec_dev, launches);
        return;
    }
    auto take = [&P]() {
        cudaEvent_t e = nullptr;
        if (!P.kev_free.empty()) {
            e = P.kev_free.back();
            P.kev_free.pop_back();
        } else {
            PW_CUDA(cudaEventCreate(&e));
        }
        return e;
    };
    Program::KernelEvent ke{B.kernel, take(), take()};
    PW_CUDA(cudaEventRecord(ke.start, P.stream));
    launch_batch_body(P, B, node, T, rec_dev, launches);
    PW_CUDA(cudaEventRecord(ke.end, P.stream));
    P.kev_pending.push_back(ke);
}

bool run_pipelined(Program& P, LaunchProgram& L, std::vector<TensorBinding>& T, uint64_t& launches) {
    PipePlan pp;
    if (!plan_pipeline(P, L, T, false, pp)) return false;
    const std::vector<Batch*>& chain = pp.chain;
    const std::vector<int>& producer = pp.producer;
    const int C = pp.C;
    const int nw = static_cast<int>(chain.size());
    auto range = [&](const Batch* B, int c, int ti, int k) {
        const int np = P.plan.kernels[B->kernel].num_tensor_params;
        return B->chunk_ranges[(static_cast<size_t>(c) * np + ti) * 2 + k];
    };
    P.timing.chunks = static_cast<uint64_t>(C);

    if (!P.h2d_stream) {
        PW_CUDA(cudaStreamCreateWithFlags(&P.h2d_stream, cudaStreamNonBlocking));
        PW_CUDA(cudaStreamCreateWithFlags(&P.d2h_stream, cudaStreamNonBlocking));
    }
    while (P.pipe_events.size() < static_cast<size_t>(2 * C + 2)) {
        cudaEvent_t e;
        PW_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        P.pipe_events.push_back(e);
    }
    cudaEvent_t ev_start = P.pipe_events[2 * C], ev_end = P.pipe_events[2 * C + 1];
    PW_CUDA(cudaEventRecord(ev_start, P.stream));  // copies wait for earlier work on the compute stream
    PW_CUDA(cudaStreamWaitEvent(P.h2d_stream, ev_start, 0));
    PW_CUDA(cudaStreamWaitEvent(P.d2h_stream, ev_start, 0));
    // inputs are copied once: the staged part of each tensor is kept one interval [lo, hi), grown on both sides
    std::vector<int64_t> staged_lo(T.size(), 0), staged_hi(T.size(), -1);
    PW_CUDA(cudaEventRecord(P.ev0, P.stream));
    for (int c = 0; c < C; ++c) {
        for (int w = 0; w < nw; ++w) {
            const Batch* B = chain[w];
            const KernelImpl& ki = P.impls[B->kernel];
            const Node& node = *B->node;
            const int np = P.plan.kernels[B->kernel].num_tensor_params;
            for (int ti = 0; ti < np; ++ti) {
                const uint32_t tid = node.tensor_args[node.param_to_arg[ti]].tensor;
                TensorBinding& tb = T[tid];
                if (tb.on_device || !ki.param_read[ti] || producer[tid] >= 0) continue;  // produced in the chain
                const size_t eb = tb.bytes / static_cast<size_t>(std::max<int64_t>(tb.span, 1));
                int64_t& s_lo = staged_lo[tid];
                int64_t& s_hi = staged_hi[tid];
                const int64_t lo = range(B, c, ti, 0), hi = range(B, c, ti, 1);
                auto copy_in = [&](int64_t a, int64_t b) {
                    if (b <= a) return;
                    PW_CUDA(cudaMemcpyAsync(tb.dev + a * eb, static_cast<char*>(tb.user_ptr) + a * eb, (b - a) * eb,
                                            cudaMemcpyHostToDevice, P.h2d_stream));
                    P.timing.h2d_bytes += (b - a) * eb;
                };
                if (s_hi < 0) {
                    copy_in(lo, hi);
                    s_lo = lo;
                    s_hi = hi;
                } else {
                    if (lo < s_lo) copy_in(lo, s_lo);  // gaps are filled so the staged part stays one interval
                    if (hi > s_hi) copy_in(s_hi, hi);
                    s_lo = std::min(s_lo, lo);
                    s_hi = std::max(s_hi, hi);
                }
            }
        }
        PW_CUDA(cudaEventRecord(P.pipe_events[2 * c], P.h2d_stream));
        PW_CUDA(cudaStreamWaitEvent(P.stream, P.pipe_events[2 * c], 0));
        for (int w = 0; w < nw; ++w) {
            const Batch* B = chain[w];
            Batch part;
            part.kernel = B->kernel;
            part.node = B->node;
            part.stride = B->stride;
            part.aligned_rows = B->aligned_rows;
            part.fast_ok = B->fast_ok;
            const int64_t t0 = B->ntasks * c / C, t1 = B->ntasks * (c + 1) / C;
            part.ntasks = t1 - t0;
            part.dev_off = B->dev_off + static_cast<size_t>(t0) * B->stride;
            launch_batch(P, part, *B->node, T, L.rec_dev, launches);
        }
        PW_CUDA(cudaEventRecord(P.pipe_events[2 * c + 1], P.stream));
        PW_CUDA(cudaStreamWaitEvent(P.d2h_stream, P.pipe_events[2 * c + 1], 0));
        for (int w = 0; w < nw; ++w) {
            const Batch* B = chain[w];
            const KernelImpl& ki = P.impls[B->kernel];
            const Node& node = *B->node;
            const int np = P.plan.kernels[B->kernel].num_tensor_params;
            for (int ti = 0; ti < np; ++ti) {
                const uint32_t tid = node.tensor_args[node.param_to_arg[ti]].tensor;
                TensorBinding& tb = T[tid];
                if (tb.on_device || !ki.param_write[ti]) continue;
                const int64_t lo = range(B, c, ti, 0), hi = range(B, c, ti, 1);
                const size_t eb = tb.bytes / static_cast<size_t>(std::max<int64_t>(tb.span, 1));
                PW_CUDA(cudaMemcpyAsync(static_cast<char*>(tb.user_ptr) + lo * eb, tb.dev + lo * eb, (hi - lo) * eb,
                                        cudaMemcpyDeviceToHost, P.d2h_stream));
                P.timing.d2h_bytes += (hi - lo) * eb;
            }
        }
    }
    PW_CUDA(cudaEventRecord(P.ev1, P.stream));
    PW_CUDA(cudaEventRecord(ev_end, P.d2h_stream));
    PW_CUDA(cudaStreamWaitEvent(P.stream, ev_end, 0));  // the run's final sync on the compute stream covers the copies
    return true;
}

}  // namespace

namespace {

// NVRTC build of the row program `tp` as kernel `name` (+ `name`_v); param types from the kernel's tile params,
// plus f32 for the params at and after `extra_f32_from` (the epilogue's scratch tile).
bool build_row_program(const dev::TileProgram& tp, const KernelDef& kd, int extra_f32_from, const std::string& name,
                       std::string* cubin, std::string* note) {
    if (!jit::row_local(tp, note)) return false;
    int types[dev::kMaxParams] = {};
    for (const auto& kp : kd.params)
        if (kp.tensor_index >= 0 && kp.tensor_index < dev::kMaxParams) types[kp.tensor_index] = ptype(kp.v.dtype);
    for (int i = extra_f32_from; i >= 0 && i < dev::kMaxParams; ++i) types[i] = dev::PT_F32;
    const std::string src = jit::gen_row_kernel(tp, types, name);
    if (const char* dir = std::getenv("PTOWSP_JIT_DUMP")) {  // keep the generated source for inspection
        std::ofstream f(std::string(dir) + "/" + name + ".cu");
        f << src;
    }
    return jit::compile_cubin(src, name, cubin, note);
}

// Slot fields an instruction of the row-local set reads or writes; false for any other op.
bool slot_fields(dev::TPInstr& in, std::vector<int*>& out) {
    out.clear();
    switch (in.op) {
        case dev::TP_LOAD: out = {&in.dst}; return true;
        case dev::TP_STORE: out = {&in.a}; return true;
        case dev::TP_MOV: case dev::TP_BINS: case dev::TP_EXP: case dev::TP_RSQRT:
        case dev::TP_ROWSUM: case dev::TP_ROWMAX: case dev::TP_ROWMEAN: out = {&in.dst, &in.a}; return true;
        case dev::TP_BIN: case dev::TP_MATMUL: out = {&in.dst, &in.a, &in.b}; return true;
        default: return false;
    }
}

}  // namespace

void jit_prepare(KernelImpl& ki, const KernelDef& kd, int k) {
    ki.jit_state = -1;
    if (!ki.tp_ok) return;
    if (build_row_program(ki.tp, kd, -1, "ptowsp_rows_k" + std::to_string(k), &ki.jit_cubin, &ki.jit_note))
        ki.jit_state = 2;
}

bool split_matmul_epilogue(KernelImpl& ki, const KernelDef& kd, int k) {
    const dev::TileProgram& tp = ki.tp;
    const int np = kd.num_tensor_params;
    if (np + 1 > dev::kMaxParams) return false;
    int mm = -1;
    for (int i = 0; i < tp.ninstr; ++i)
        if (tp.ins[i].op == dev::TP_MATMUL) {
            if (mm >= 0) return false;  // one contraction per kernel
            mm = i;
        }
    if (mm < 0) return false;
    const dev::TPInstr& m = tp.ins[mm];
    // the shapes of the tcgen05 tile kernel: 128 rows, 64/128/256 columns, K a multiple of 64
    if (m.rows != 128 || !(m.cols == 64 || m.cols == 128 || m.cols == 256) || m.k < 64 || m.k % 64) return false;
    if (tp.slots[m.dst].word != dev::W_F32) return false;
    int la = -1, lb = -1;
    for (int i = 0; i < mm; ++i) {
        if (tp.ins[i].op != dev::TP_LOAD) continue;
        if (tp.ins[i].dst == m.a) la = i;
        if (tp.ins[i].dst == m.b) lb = i;
    }
    if (la < 0 || lb < 0 || la == lb) return false;
    const int pa = tp.ins[la].param, pb = tp.ins[lb].param;
    auto param_dtype = [&](int ti) {
        for (const auto& kp : kd.params)
            if (kp.tensor_index == ti) return kp.v.dtype;
        return DType::F32;
    };
    if (pa == pb || param_dtype(pa) != DType::F16 || param_dtype(pb) != DType::F16) return false;
    // the operand tiles and their params serve the matmul alone
    std::vector<int*> f;
    dev::TileProgram ep{};
    ep.ninstr = 0;
    for (int i = 0; i < tp.ninstr; ++i) {
        if (i == la || i == lb) continue;
        dev::TPInstr in = tp.ins[i];
        if (i == mm) {
            dev::TPInstr ld{};
            ld.op = dev::TP_LOAD;
            ld.dst = m.dst;
            ld.param = np;  // the scratch tile
            ld.rows = m.rows;
            ld.cols = m.cols;
            in = ld;
        } else {
            if (!slot_fields(in, f)) return false;
            for (int* x : f)
                if (*x == m.a || *x == m.b) return false;
            if ((in.op == dev::TP_LOAD || in.op == dev::TP_STORE) && (in.param == pa || in.param == pb)) return false;
        }
        ep.ins[ep.ninstr++] = in;
    }
    // keep only the slots the epilogue uses, renumbered in order
    std::vector<int> remap(tp.nslots, -1);
    ep.nslots = 0;
    for (int i = 0; i < ep.ninstr; ++i) {
        slot_fields(ep.ins[i], f);
        for (int* x : f) {
            if (*x < 0 || *x >= tp.nslots) return false;
            if (remap[*x] < 0) {
                remap[*x] = ep.nslots;
                ep.slots[ep.nslots++] = tp.slots[*x];
            }
            *x = remap[*x];
        }
    }
    for (int i = 0; i < dev::kMaxParams; ++i) ep.scalar_types[i] = tp.scalar_types[i];
    ep.smem_words = 0;
    std::string cubin, note;
    if (!build_row_program(ep, kd, np, "ptowsp_ep_k" + std::to_string(k), &cubin, &note)) return false;
    ki.ep_tp = ep;
    ki.ep_a = pa;
    ki.ep_b = pb;
    ki.ep_n = m.cols;
    ki.ep_k = m.k;
    ki.ep_cubin = std::move(cubin);
    ki.ep_jit_state = 2;
    ki.kind = ImplKind::MatmulEpilogue;
    ki.jit_note = "matmul on tcgen05, the rest as a fused row program";
    return true;
}

bool build_stage_program(const dev::TileProgram& tp, const KernelDef& kd, const std::string& name, std::string* cubin,
                         std::string* note) {
    return build_row_program(tp, kd, kd.num_tensor_params, name, cubin, note);
}

bool match_attention(KernelImpl& ki, const KernelDef& kd) {
    // value id -> the kernel param it is (through Load ops), and the Constant ops' values
    std::map<int, const KernelParam*> param_of;
    for (const auto& kp : kd.params) param_of[kp.id] = &kp;
    std::map<int, double> constant;
    std::vector<const OpInfo*> seq;
    for (const auto& op : kd.ops) {
        if (op.kind == "Constant" && op.result >= 0) {
            const json::Value* v = op.attrs.get("value");
            if (!v) return false;
            constant[op.result] = v->as_f64();
        } else if (op.kind == "Load" && op.result >= 0 && op.operands.size() == 1 && param_of.count(op.operands[0])) {
            param_of[op.result] = param_of[op.operands[0]];
        } else {
            seq.push_back(&op);
        }
    }
    auto tensor = [&](int id) -> const KernelParam* {
        auto it = param_of.find(id);
        return it != param_of.end() && it->second->tensor_index >= 0 ? it->second : nullptr;
    };
    auto is_op = [&](size_t i, const char* kind, size_t nops) {
        return i < seq.size() && seq[i]->kind == kind && seq[i]->operands.size() == nops &&
               (nops == 0 || seq[i]->result >= 0 || std::string(kind) == "Store");
    };
    size_t i = 0;
    if (!is_op(i, "Matmul", 2)) return false;
    const KernelParam* q = tensor(seq[i]->operands[0]);
    const KernelParam* kt = tensor(seq[i]->operands[1]);
    int s = seq[i++]->result;
    int mode = 0, sidx = -1;
    double sconst = 1.0;
    if (is_op(i, "Mul", 2)) {  // S * scale: a scalar param or a constant, on either side
        const int a = seq[i]->operands[0], b = seq[i]->operands[1];
        const int other = a == s ? b : (b == s ? a : -1);
        if (other < 0) return false;
        auto pit = param_of.find(other);
        if (pit != param_of.end() && pit->second->scalar_index >= 0 && pit->second->v.dtype == DType::F32) {
            mode = 2;
            sidx = pit->second->scalar_index;
        } else if (constant.count(other)) {
            mode = 1;
            sconst = constant[other];
        } else {
            return false;
        }
        s = seq[i++]->result;
    }
    if (!is_op(i, "RowMax", 1) || seq[i]->operands[0] != s) return false;
    const int m = seq[i++]->result;
    if (!is_op(i, "Sub", 2) || seq[i]->operands[0] != s || seq[i]->operands[1] != m) return false;
    const int d = seq[i++]->result;
    if (!is_op(i, "Exp", 1) || seq[i]->operands[0] != d) return false;
    const int e = seq[i++]->result;
    if (!is_op(i, "RowSum", 1) || seq[i]->operands[0] != e) return false;
    const int l = seq[i++]->result;
    if (!is_op(i, "Div", 2) || seq[i]->operands[0] != e || seq[i]->operands[1] != l) return false;
    const int w = seq[i++]->result;
    if (!is_op(i, "Matmul", 2) || seq[i]->operands[0] != w) return false;
    const KernelParam* v = tensor(seq[i]->operands[1]);
    const int o = seq[i++]->result;
    if (!is_op(i, "Store", 2) || seq[i]->operands[1] != o) return false;
    const KernelParam* out = tensor(seq[i++]->operands[0]);
    if (i != seq.size() || !q || !kt || !v || !out) return false;
    const int L = kt->v.cols;
    auto shape = [](const KernelParam* p, DType t, int r, int c) { return p->v.dtype == t && p->v.rows == r && p->v.cols == c; };
    if (!shape(q, DType::F16, 128, 128) || !shape(kt, DType::F16, 128, L) || !shape(v, DType::F32, L, 128) ||
        !shape(out, DType::F32, 128, 128) || L < 64 || L % 64 != 0)
        return false;
    // the inputs are read only, the output written only (the one Store)
    if (ki.param_write[q->tensor_index] || ki.param_write[kt->tensor_index] || ki.param_write[v->tensor_index] ||
        out == q || out == kt || out == v)
        return false;
    for (int id : {s, m, d, e, l, w, o}) {
        auto it = kd.values.find(id);
        if (it == kd.values.end() || it->second.dtype != DType::F32) return false;
    }
    ki.at_q = q->tensor_index;
    ki.at_kt = kt->tensor_index;
    ki.at_v = v->tensor_index;
    ki.at_o = out->tensor_index;
    ki.at_L = L;
    ki.at_scale_mode = mode;
    ki.at_scale_index = sidx;
    ki.at_scale_const = static_cast<float>(sconst);
    return true;
}

bool split_stages(KernelImpl& ki, const KernelDef& kd) {
    const dev::TileProgram& tp = ki.tp;
    const int np = kd.num_tensor_params;
    const int nslots = tp.nslots;
    std::vector<int> def(nslots, -1);  // defining instruction of each slot (one at most)
    std::vector<int*> f;
    int nmm = 0;
    for (int i = 0; i < tp.ninstr; ++i) {
        dev::TPInstr in = tp.ins[i];
        if (!slot_fields(in, f)) return false;  // ops without a row form (iota, sort, extract)
        if (in.op == dev::TP_MATMUL) ++nmm;
        if (in.op == dev::TP_STORE) continue;
        if (in.dst < 0 || in.dst >= nslots || def[in.dst] >= 0) return false;
        def[in.dst] = i;
    }
    if (nmm == 0) return false;
    auto param_dtype = [&](int ti) {
        for (const auto& kp : kd.params)
            if (kp.tensor_index == ti) return kp.v.dtype;
        return DType::F32;
    };
    // stage of each instruction: row stages 0, 2, 4, ... around matmul stages 1, 3, ...
    std::vector<int> stage_of(tp.ninstr);
    int st = 0;
    for (int i = 0; i < tp.ninstr; ++i) {
        if (tp.ins[i].op == dev::TP_MATMUL) {
            stage_of[i] = st | 1;
            st = (st | 1) + 1;
        } else {
            stage_of[i] = st;
        }
    }
    const int nstages = st + 1;
    // a slot loaded straight from a param (no transposed load) is re-read from the param wherever it is needed --
    // unless the kernel stores to that param, when a later stage would read the stored values instead
    std::vector<char> stored(dev::kMaxParams, 0);
    for (int i = 0; i < tp.ninstr; ++i)
        if (tp.ins[i].op == dev::TP_STORE && tp.ins[i].param >= 0 && tp.ins[i].param < dev::kMaxParams)
            stored[tp.ins[i].param] = 1;
    auto param_load = [&](int slot) {
        const int d = def[slot];
        return d >= 0 && tp.ins[d].op == dev::TP_LOAD && tp.ins[d].k == 0 && !stored[tp.ins[d].param] ? d : -1;
    };
    // uses of each slot by stage
    std::vector<std::vector<int>> used_in(nslots);
    for (int i = 0; i < tp.ninstr; ++i) {
        dev::TPInstr in = tp.ins[i];
        slot_fields(in, f);
        for (size_t j = (in.op == dev::TP_STORE ? 0 : 1); j < f.size(); ++j) used_in[*f[j]].push_back(stage_of[i]);
    }
    // matmul operands: the param itself when the slot is a plain param load of the operand's shape
    std::vector<Stage> stages;
    std::vector<int> scratch_of(nslots, -1);
    std::vector<std::pair<int, int>> scratch;
    auto need_scratch = [&](int slot) {
        if (scratch_of[slot] < 0) {
            scratch_of[slot] = static_cast<int>(scratch.size());
            scratch.emplace_back(tp.slots[slot].rows, tp.slots[slot].cols);
        }
        return scratch_of[slot];
    };
    for (int i = 0; i < tp.ninstr; ++i) {
        const dev::TPInstr& in = tp.ins[i];
        if (in.op != dev::TP_MATMUL) continue;
        if (tp.slots[in.dst].word != dev::W_F32 || tp.slots[in.a].word != dev::W_F32 ||
            tp.slots[in.b].word != dev::W_F32)
            return false;
        Stage S;
        S.mm = true;
        S.m = in.rows;
        S.n = in.cols;
        S.k = in.k;
        const int la = param_load(in.a), lb = param_load(in.b);
        const bool pa = la >= 0 && tp.ins[la].rows == S.m && tp.ins[la].cols == S.k;
        const bool pb = lb >= 0 && tp.ins[lb].rows == S.k && tp.ins[lb].cols == S.n;
        S.a = pa ? tp.ins[la].param : ~need_scratch(in.a);
        S.b = pb ? tp.ins[lb].param : ~need_scratch(in.b);
        S.c = need_scratch(in.dst);
        S.tc = pa && pb && S.a != S.b && param_dtype(S.a) == DType::F16 && param_dtype(S.b) == DType::F16 &&
               S.m == 128 && S.n % 64 == 0 && S.k >= 64 && S.k % 64 == 0;
        S.tn = S.n % 256 == 0 ? 256 : (S.n % 128 == 0 ? 128 : 64);
        S.rows = stage_of[i];  // the stage number until the list is assembled
        stages.push_back(S);
    }
    // values crossing from a row stage to a later stage (other than plain param loads, which are re-read)
    for (int sl = 0; sl < nslots; ++sl) {
        if (def[sl] < 0 || tp.ins[def[sl]].op == dev::TP_MATMUL) continue;
        const int ds = stage_of[def[sl]];
        bool later = false;
        for (int u : used_in[sl]) later = later || u > ds;
        if (later && param_load(sl) < 0) need_scratch(sl);
    }
    if (np + static_cast<int>(scratch.size()) > dev::kMaxParams) return false;
    for (int sl = 0; sl < nslots; ++sl)  // scratch tiles hold f32 values only
        if (scratch_of[sl] >= 0 && tp.slots[sl].word != dev::W_F32) return false;
    // row stages: the stage's own instructions, led by loads of what earlier stages left in scratch or in params,
    // followed by stores of what later stages need
    std::vector<Stage> out;
    size_t next_mm = 0;
    for (int sg = 0; sg < nstages; ++sg) {
        if (sg & 1) {
            out.push_back(stages[next_mm++]);
            continue;
        }
        dev::TileProgram rp{};
        rp.ninstr = 0;
        std::vector<char> have(nslots, 0);
        auto emit = [&](const dev::TPInstr& x) {
            if (rp.ninstr >= dev::kTPMaxInstr) return false;
            rp.ins[rp.ninstr++] = x;
            return true;
        };
        auto bring = [&](int slot) {  // make an earlier stage's value available in this stage
            if (have[slot]) return true;
            have[slot] = 1;
            const int pl = param_load(slot);
            if (pl >= 0) return emit(tp.ins[pl]);
            if (scratch_of[slot] < 0) return false;
            dev::TPInstr ld{};
            ld.op = dev::TP_LOAD;
            ld.dst = slot;
            ld.param = np + scratch_of[slot];
            ld.rows = tp.slots[slot].rows;
            ld.cols = tp.slots[slot].cols;
            return emit(ld);
        };
        bool any = false;  // an instruction besides re-reads of params for matmuls
        for (int i = 0; i < tp.ninstr; ++i) {
            if (stage_of[i] != sg) continue;
            dev::TPInstr in = tp.ins[i];
            slot_fields(in, f);
            for (size_t j = (in.op == dev::TP_STORE ? 0 : 1); j < f.size(); ++j)
                if (def[*f[j]] < 0 || stage_of[def[*f[j]]] < sg)
                    if (!bring(*f[j])) return false;
            if (in.op == dev::TP_LOAD && param_load(in.dst) == i) {
                // a param load is emitted where a row op of this stage uses it (or a later stage needs it in
                // scratch); loads only the matmuls read are dropped
                bool row_use = scratch_of[in.dst] >= 0;
                for (int u : used_in[in.dst]) row_use = row_use || (u == sg);
                if (!row_use) continue;
                have[in.dst] = 1;
            } else if (in.op != dev::TP_STORE) {
                have[in.dst] = 1;
            }
            if (!emit(in)) return false;
            any = true;
        }
        for (int sl = 0; sl < nslots; ++sl)  // values of this stage that later stages read from scratch
            if (def[sl] >= 0 && stage_of[def[sl]] == sg && scratch_of[sl] >= 0 && tp.ins[def[sl]].op != dev::TP_MATMUL) {
                dev::TPInstr stv{};
                stv.op = dev::TP_STORE;
                stv.a = sl;
                stv.param = np + scratch_of[sl];
                stv.rows = tp.slots[sl].rows;
                stv.cols = tp.slots[sl].cols;
                if (!emit(stv)) return false;
                any = true;
            }
        if (!any) continue;
        // keep only the slots the stage uses, renumbered in order
        std::vector<int> remap(nslots, -1);
        rp.nslots = 0;
        for (int i = 0; i < rp.ninstr; ++i) {
            slot_fields(rp.ins[i], f);
            for (int* x : f) {
                if (remap[*x] < 0) {
                    remap[*x] = rp.nslots;
                    rp.slots[rp.nslots++] = tp.slots[*x];
                }
                *x = remap[*x];
            }
        }
        for (int i = 0; i < dev::kMaxParams; ++i) rp.scalar_types[i] = tp.scalar_types[i];
        rp.smem_words = 0;
        std::string why;
        if (!jit::row_local(rp, &why)) return false;
        Stage S;
        S.tp = rp;
        S.rows = jit::program_rows(rp);
        out.push_back(S);
    }
    ki.stages = std::move(out);
    ki.scratch_tiles = std::move(scratch);
    return true;
}

// After a walk: when the workload is one loop over a ragged axis or a sparse selection with one task as its body
// (the reference's ParallelFor over Ragged, pto_codegen.cpp:2305-2416, and Select, :2417-2457), and its task
// records are affine in the loop variable, keep what a later run with other lengths or another selection needs
// to rebuild them on the device.  Only kernels whose launch reads nothing but the records qualify (row programs,
// row kernels, the tile-program interpreter), with round-robin or no dispatch (the makespan is then recomputed
// from the task count alone).
void plan_expand(Program& P, LaunchProgram& L, const std::vector<Walker::LoopNote>& loops) {
    if (loops.size() != 1 || L.waves.size() != 1 || L.waves[0].batches.size() != 1) return;
    const auto& ln = loops[0];
    if (ln.node != P.plan.body.get()) return;
    Batch& B = L.waves[0].batches[0];
    if (B.node != ln.node->body.get() || B.sel || B.ntasks < 2 || B.rec.empty()) return;
    const KernelImpl& ki = P.impls[B.kernel];
    if (ki.kind != ImplKind::TileProgram && ki.kind != ImplKind::RmsNorm && ki.kind != ImplKind::Softmax) return;
    const std::string& pol = P.plan.schedule.dispatch_policy;
    if (!pol.empty() && pol != "round_robin" && pol != "work_steal") return;
    // exactly one data-dependent key entry, this loop's
    size_t idx = SIZE_MAX;
    for (size_t i = 0; i + 1 < L.key.size(); ++i) {
        const char k = L.key[i][0];
        if (k != 'r' && k != 'c') continue;
        if (idx != SIZE_MAX || L.key[i].compare(0, ln.key_name.size() + 1, ln.key_name + "=") != 0) return;
        idx = i;
    }
    if (idx == SIZE_MAX) return;
    const int64_t n = B.ntasks, stride = B.stride;
    auto var = [&](int64_t t) { return ln.kind == 'r' ? t : ln.vars[static_cast<size_t>(t)]; };
    if (ln.kind == 'c' && static_cast<int64_t>(ln.vars.size()) != n) return;
    int64_t t1 = 1;
    while (t1 < n && var(t1) == var(0)) ++t1;
    if (t1 >= n) return;
    std::vector<int64_t> base(static_cast<size_t>(stride)), delta(static_cast<size_t>(stride));
    const int64_t dv = var(t1) - var(0);
    for (int64_t w = 0; w < stride; ++w) {
        const int64_t d = B.rec[t1 * stride + w] - B.rec[w];
        if (d % dv) return;
        delta[w] = d / dv;
        base[w] = B.rec[w] - var(0) * delta[w];
    }
    for (int64_t t = 0; t < n; ++t)
        for (int64_t w = 0; w < stride; ++w)
            if (B.rec[t * stride + w] != base[w] + var(t) * delta[w]) return;
    for (int w = 0; w < P.plan.kernels[B.kernel].num_tensor_params; ++w)
        if ((base[w] & 3) || (delta[w] & 3)) B.aligned_rows = false;  // some var may give an unaligned view
    auto X = std::make_unique<LoopExpand>();
    X->kind = ln.kind;
    X->key_index = idx;
    X->key_name = ln.key_name;
    const uint64_t outer_sym = ln.kind == 'r' ? ln.node->axis.outer_sym : ln.node->outer_sym;
    const std::string outer_name = "s" + std::to_string(outer_sym) + "=";
    for (size_t i = 0; i + 1 < L.key.size(); ++i)
        if (L.key[i].compare(0, outer_name.size(), outer_name) == 0) X->outer_key_index = i;
    X->parallel = ln.node->kind != Node::Kind::ForEach;
    if (ln.kind == 'r') {
        X->lengths_sym = ln.node->axis.lengths_sym;
        X->outer_sym = ln.node->axis.outer_sym;
    } else {
        X->indptr_sym = ln.node->indptr_sym;
        X->indices_sym = ln.node->indices_sym;
        X->outer_sym = ln.node->outer_sym;
    }
    for (uint8_t w : ki.param_write) X->writes = X->writes || w;
    X->base = base;
    X->delta = delta;
    std::vector<int64_t> bd(base);
    bd.insert(bd.end(), delta.begin(), delta.end());
    PW_CUDA(cudaMalloc(&X->base_delta_dev, bd.size() * sizeof(int64_t)));
    PW_CUDA(cudaMemcpy(X->base_delta_dev, bd.data(), bd.size() * sizeof(int64_t), cudaMemcpyHostToDevice));
    L.expand = std::move(X);
}

// A run whose only changed runtime answer is the expandable loop's: rebuild its task records on the device from
// the new count (ragged: the sum of the lengths; selection: the indices, uploaded), recompute the makespan with the
// same Scheduler::issue model over that many tasks, and keep the cached table.  False (nothing changed) when the
// new run does not fit: no task, or a selection that repeats an index while the kernel writes (its tasks would
// conflict: the host walk orders them).
bool expand_on_device(Program& P, LaunchProgram& L, RuntimeContext* ctx, size_t ntensors) {
    LoopExpand& X = *L.expand;
    auto sym_u64 = [&](uint64_t id) { return ctx->get_symbol_u64 ? ctx->get_symbol_u64(ctx->ctx, id) : 0; };
    auto sym_ptr = [&](uint64_t id) {
        return ctx->get_symbol_ptr ? static_cast<const int32_t*>(ctx->get_symbol_ptr(ctx->ctx, id)) : nullptr;
    };
    int64_t n = 0;
    uint64_t key_value = 0;
    const int32_t* vars = nullptr;
    const int64_t outer = static_cast<int64_t>(sym_u64(X.outer_sym));
    if (X.kind == 'r') {
        const int32_t* lens = sym_ptr(X.lengths_sym);
        if (!lens) return false;
        for (int64_t i = 0; i < outer; ++i) n += lens[i];
        key_value = static_cast<uint64_t>(n);
    } else {
        const int32_t* indptr = sym_ptr(X.indptr_sym);
        vars = sym_ptr(X.indices_sym);
        if (!indptr || !vars) return false;
        n = indptr[outer];
        key_value = csr_hash(indptr, vars, outer);
        if (X.writes) {
            std::unordered_set<int32_t> seen;
            for (int64_t p = 0; p < n; ++p)
                if (!seen.insert(vars[p]).second) return false;
        }
    }
    if (n < 1) return false;
    Batch& B = L.waves[0].batches[0];
    const size_t need = static_cast<size_t>(n) * static_cast<size_t>(B.stride);
    if (need > L.rec_cap) {
        int64_t* nb = nullptr;
        PW_CUDA(cudaStreamSynchronize(P.stream));  // earlier runs may still read the old table
        PW_CUDA(cudaMalloc(&nb, need * sizeof(int64_t)));
        if (L.rec_dev) PW_CUDA(cudaFree(L.rec_dev));
        L.rec_dev = nb;
        L.rec_cap = need;
    }
    const int32_t* vars_dev = nullptr;
    if (vars) {
        if (X.vars_cap < static_cast<size_t>(n)) {
            PW_CUDA(cudaStreamSynchronize(P.stream));
            if (X.vars_dev) PW_CUDA(cudaFree(X.vars_dev));
            X.vars_dev = nullptr;
            PW_CUDA(cudaMalloc(&X.vars_dev, static_cast<size_t>(n) * sizeof(int32_t)));
            X.vars_cap = static_cast<size_t>(n);
        }
        PW_CUDA(cudaMemcpyAsync(X.vars_dev, vars, static_cast<size_t>(n) * sizeof(int32_t), cudaMemcpyHostToDevice,
                                P.stream));
        PW_CUDA(cudaStreamSynchronize(P.stream));  // the indices are the caller's memory
        vars_dev = X.vars_dev;
    }
    PW_CUDA(dev::launch_expand_records(L.rec_dev, B.stride, n, X.base_delta_dev, vars_dev, P.stream));
    B.ntasks = n;
    B.dev_off = 0;
    L.rec_elems = need;
    L.tasks = static_cast<uint64_t>(n);
    // makespan: the walk's Scheduler::issue sequence for n tasks of this kernel (pto_codegen.cpp:2679-2692)
    const Schedule& sc = P.plan.schedule;
    Scheduler sched(static_cast<uint32_t>(sc.num_targets > 0 ? sc.num_targets : (sc.streams > 0 ? sc.streams : 1)),
                    static_cast<uint64_t>(sc.window_tasks));
    const uint64_t cyc = P.impls[B.kernel].cycles;
    uint64_t done = 0, cur = 0;
    for (int64_t t = 0; t < n; ++t) {
        const uint32_t wid = sc.dispatch_policy.empty() ? 0u : static_cast<uint32_t>(static_cast<uint64_t>(t) % sched.n);
        if (X.parallel) done = std::max(done, sched.issue(cyc, wid, 0));
        else cur = sched.issue(cyc, wid, cur);
    }
    L.makespan = X.parallel ? done : cur;
    L.key[X.key_index] = X.key_name + "=" + std::to_string(key_value);
    if (X.outer_key_index != SIZE_MAX)
        L.key[X.outer_key_index] = "s" + std::to_string(X.outer_sym) + "=" + std::to_string(static_cast<uint64_t>(outer));
    // which elements the loop writes changed: stage every host tensor in and out
    L.full_write.assign(ntensors, 0);
    L.write_first.assign(ntensors, 0);
    L.no_pipeline = true;
    return true;
}

// The workload's CSP pipeline as one CTA per process (dev::launch_csp_pipeline).  Uploads the operations, records and
// programs at the first launch; every launch builds the slots' tensor params from the current bindings and zeroes
// the channel counters.  False (nothing launched) when the processes cannot all be resident at once.
bool launch_csp(Program& P, LaunchProgram& L, std::vector<TensorBinding>& T, uint64_t& launches) {
    CspDevice& D = *L.csp;
    const size_t nslot = D.slot_node.size(), nchan = D.caps.size();
    const int nproc = static_cast<int>(D.proc_first.size()) - 1;
    if (!D.ops_dev) {
        auto up = [&](auto** dst, const auto& v) {
            using E = typename std::decay_t<decltype(v)>::value_type;
            const size_t bytes = std::max<size_t>(v.size(), 1) * sizeof(E);
            PW_CUDA(cudaMalloc(reinterpret_cast<void**>(dst), bytes));
            if (!v.empty())
                PW_CUDA(cudaMemcpyAsync(*dst, v.data(), v.size() * sizeof(E), cudaMemcpyHostToDevice, P.stream));
        };
        up(&D.ops_dev, D.ops);
        up(&D.first_dev, D.proc_first);
        up(&D.rec_dev, D.rec);
        up(&D.caps_dev, D.caps);
        std::vector<const dev::TileProgram*> progs;
        for (const Node* n : D.slot_node) progs.push_back(P.impls[n->kernel_index].tp_dev);
        up(&D.prog_dev, progs);
        PW_CUDA(cudaMalloc(&D.tb_dev, std::max<size_t>(nslot, 1) * sizeof(dev::TaskBatch)));
        PW_CUDA(cudaMalloc(&D.counts_dev, std::max<size_t>(2 * nchan, 1) * sizeof(unsigned)));
        PW_CUDA(cudaStreamSynchronize(P.stream));  // the host vectors stay; the copies must not race a later change
    }
    std::vector<dev::TaskBatch> tbs(nslot);
    for (size_t k = 0; k < nslot; ++k) {
        bool rows_ok = true;
        fill_task_params(P, D.slot_node[k]->kernel_index, *D.slot_node[k], T, tbs[k], rows_ok);
        tbs[k].rec = D.rec_dev;
        tbs[k].ntasks = 0;
    }
    if (nslot)
        PW_CUDA(cudaMemcpyAsync(D.tb_dev, tbs.data(), nslot * sizeof(dev::TaskBatch), cudaMemcpyHostToDevice, P.stream));
    if (nchan) PW_CUDA(cudaMemsetAsync(D.counts_dev, 0, 2 * nchan * sizeof(unsigned), P.stream));
    dev::CspArgs a{};
    a.ops = D.ops_dev;
    a.proc_first = D.first_dev;
    a.batches = D.tb_dev;
    a.progs = D.prog_dev;
    a.counts = D.counts_dev;
    a.caps = D.caps_dev;
    a.nproc = nproc;
    a.nchan = static_cast<int>(nchan);
    a.err = P.err_dev;
    cudaError_t e = cudaSuccess;
    if (!dev::launch_csp_pipeline(a, D.smem, P.stream, &e)) {
        if (nslot) PW_CUDA(cudaStreamSynchronize(P.stream));  // the param copy reads `tbs`
        return false;
    }
    if (e != cudaSuccess) throw Error(PTOWSP_ERR_CUDA, std::string("CSP pipeline launch: ") + cudaGetErrorString(e));
    launches++;
    if (nslot) PW_CUDA(cudaStreamSynchronize(P.stream));  // `tbs` is a host temporary of the param copy
    return true;
}

uint64_t run_program(Program& P, RuntimeContext* ctx) {
    auto t_start = std::chrono::steady_clock::now();
    if (!ctx) throw Error(PTOWSP_ERR_ARG, "RuntimeContext is null");
    const bool dry = P.opt_dry != 0;  // host-only walk: no CUDA calls at all
    if (!dry) {
        PW_CUDA(cudaSetDevice(P.device));
        ensure_device_state(P);
    }
    P.timing = ptowsp_timing{};
    const Plan& plan = P.plan;

    // ---- bind tensors ----
    std::vector<TensorBinding> T(plan.tensors.size());
    bool all_device = true;
    for (size_t tid = 0; tid < plan.tensors.size(); ++tid) {
        TensorBinding& b = T[tid];
        const TensorInfo& ti = plan.tensors[tid];
        b.user_ptr = ctx->get_tensor_ptr ? ctx->get_tensor_ptr(ctx->ctx, static_cast<uint32_t>(tid)) : nullptr;
        b.strides.resize(ti.shape.size());
        int64_t span = 1;
        for (size_t d = 0; d < ti.shape.size(); ++d) {
            b.strides[d] = ctx->get_tensor_stride ? static_cast<int64_t>(ctx->get_tensor_stride(ctx->ctx, static_cast<uint32_t>(tid), static_cast<uint32_t>(d))) : 0;
            if (b.strides[d] < 0) throw Error(PTOWSP_ERR_ARG, "negative tensor strides are not supported");
            if (ti.shape[d] <= 0) span = 0;
            else if (span > 0) span += (ti.shape[d] - 1) * b.strides[d];
        }
        b.span = span;
        b.bytes = static_cast<size_t>(span) * dtype_bytes(ti.dtype);
        if (!b.user_ptr && b.bytes) throw Error(PTOWSP_ERR_ARG, "tensor " + std::to_string(tid) + " has no data pointer");
        cudaPointerAttributes attr{};
        if (!dry && b.user_ptr && cudaPointerGetAttributes(&attr, b.user_ptr) == cudaSuccess &&
            (attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged)) {
            b.on_device = true;
            b.dev = static_cast<char*>(b.user_ptr);
        }
        if (!dry) cudaGetLastError();
        if (!b.on_device && b.bytes) all_device = false;
    }
    // read / written sets per tensor from the kernels' param sets
    std::function<void(const Node&)> mark = [&](const Node& n) {
        switch (n.kind) {
            case Node::Kind::ParallelFor: case Node::Kind::ForEach: case Node::Kind::Select:
            case Node::Kind::Send: case Node::Kind::Consume: mark(*n.body); break;
            case Node::Kind::Combine: case Node::Kind::Sequential: case Node::Kind::Pipeline:
                for (auto& c : n.children) mark(*c);
                break;
            case Node::Kind::Cond: mark(*n.then_n); mark(*n.else_n); break;
            case Node::Kind::Task: {
                const KernelImpl& ki = P.impls[n.kernel_index];
                for (size_t ti = 0; ti < n.param_to_arg.size(); ++ti) {
                    auto& b = T[n.tensor_args[n.param_to_arg[ti]].tensor];
                    if (ki.param_read[ti]) b.read = true;
                    if (ki.param_write[ti]) b.written = true;
                }
                break;
            }
            case Node::Kind::SlotLoad: T[n.slot_tensor.tensor].read = true; break;
            default: break;
        }
    };
    mark(*plan.body);
    // host staging buffers
    if (P.dev_bufs.size() < T.size()) {
        P.dev_bufs.resize(T.size(), nullptr);
        P.dev_caps.resize(T.size(), 0);
    }
    for (size_t tid = 0; tid < T.size() && !dry; ++tid) {
        TensorBinding& b = T[tid];
        if (b.on_device || b.bytes == 0) continue;
        if (P.dev_caps[tid] < b.bytes) {
            if (P.dev_bufs[tid]) PW_CUDA(cudaFree(P.dev_bufs[tid]));
            P.dev_bufs[tid] = nullptr;
            P.dev_caps[tid] = 0;
            PW_CUDA(cudaMalloc(&P.dev_bufs[tid], b.bytes));
            P.dev_caps[tid] = b.bytes;
        }
        b.dev = P.dev_bufs[tid];
    }
    const bool async_run = !P.opt_sync && all_device;

    // ---- replay check for static workloads ----
    std::string stride_sig = "#";
    for (auto& b : T)
        for (auto s : b.strides) stride_sig += std::to_string(s) + ",";
    bool replay = false;
    size_t mismatches = 0, loop_mismatches = 0;
    if (P.cacheable && P.opt_cache && P.cached) {
        replay = !P.cached->key.empty() && P.cached->key.back() == stride_sig;
        for (size_t i = 0; replay && i + 1 < P.cached->key.size(); ++i) {
            const std::string& q = P.cached->key[i];
            const char kind = q[0];
            size_t eq = q.find('=');
            std::string name = q.substr(1, eq - 1);
            uint64_t want = std::stoull(q.substr(eq + 1));
            uint64_t got = 0;
            auto sym_u64 = [&](uint64_t id) { return ctx->get_symbol_u64 ? ctx->get_symbol_u64(ctx->ctx, id) : 0; };
            auto sym_ptr = [&](uint64_t id) {
                return ctx->get_symbol_ptr ? static_cast<const int32_t*>(ctx->get_symbol_ptr(ctx->ctx, id)) : nullptr;
            };
            if (kind == 's') {
                got = sym_u64(std::stoull(name));
            } else if (kind == 'a') {
                got = static_cast<uint64_t>(ctx->get_axis_size ? ctx->get_axis_size(ctx->ctx, name.c_str()) : 0);
            } else if (kind == 'r') {  // ragged axis: the sum of its lengths
                const size_t c = name.find(':');
                const int32_t* lens = sym_ptr(std::stoull(name.substr(0, c)));
                const int64_t outer = static_cast<int64_t>(sym_u64(std::stoull(name.substr(c + 1))));
                int64_t ub = 0;
                for (int64_t i = 0; lens && i < outer; ++i) ub += lens[i];
                got = static_cast<uint64_t>(ub);
            } else if (kind == 'c') {  // CSR selection: its arrays' contents
                const size_t c1 = name.find(':'), c2 = name.find(':', c1 + 1);
                got = csr_hash(sym_ptr(std::stoull(name.substr(0, c1))), sym_ptr(std::stoull(name.substr(c1 + 1, c2 - c1 - 1))),
                               static_cast<int64_t>(sym_u64(std::stoull(name.substr(c2 + 1)))));
            } else {
                replay = false;
            }
            if (got != want) {
                ++mismatches;
                const LoopExpand* X = P.cached->expand.get();
                if (X && (i == X->key_index || i == X->outer_key_index)) ++loop_mismatches;
            }
        }
        if (mismatches) {
            // only the expandable loop's ragged lengths or selection changed: rebuild its records on the device
            const bool one_loop = replay && mismatches == loop_mismatches && !dry;
            replay = one_loop && expand_on_device(P, *P.cached, ctx, T.size());
            if (replay) P.timing.expansions = 1;
        }
    }

    std::unique_ptr<LaunchProgram> fresh;
    LaunchProgram* L = nullptr;
    std::vector<std::string> log;
    uint64_t launches = 0;
    size_t launched_waves = 0;
    std::unique_ptr<Walker> W;

    auto upload_and_launch = [&](size_t upto) {
        size_t need = L->rec_elems;
        for (size_t wi = launched_waves; wi < upto; ++wi)
            for (auto& b : L->waves[wi].batches) need += b.rec.size();
        if (need > L->rec_cap) {
            int64_t* nb = nullptr;
            size_t cap = std::max<size_t>(need, L->rec_cap * 2);
            PW_CUDA(cudaMalloc(&nb, cap * sizeof(int64_t)));
            if (L->rec_dev) {
                PW_CUDA(cudaMemcpyAsync(nb, L->rec_dev, L->rec_elems * sizeof(int64_t), cudaMemcpyDeviceToDevice, P.stream));
                PW_CUDA(cudaStreamSynchronize(P.stream));
                PW_CUDA(cudaFree(L->rec_dev));
            }
            L->rec_dev = nb;
            L->rec_cap = cap;
        }
        for (size_t wi = launched_waves; wi < upto; ++wi)
            for (auto& b : L->waves[wi].batches) {
                b.dev_off = L->rec_elems;
                if (!b.rec.empty())
                    PW_CUDA(cudaMemcpyAsync(L->rec_dev + b.dev_off, b.rec.data(), b.rec.size() * sizeof(int64_t),
                                            cudaMemcpyHostToDevice, P.stream));
                L->rec_elems += b.rec.size();
            }
        for (size_t wi = launched_waves; wi < upto; ++wi)
            for (auto& b : L->waves[wi].batches) launch_batch(P, b, *b.node, T, L->rec_dev, launches);
        launched_waves = upto;
    };

    // ---- static workloads: walk before staging (the walk knows which outputs are fully overwritten) ----
    if (replay) {
        L = P.cached.get();
    } else if (P.cacheable) {
        fresh = std::make_unique<LaunchProgram>();
        L = fresh.get();
        W = std::make_unique<Walker>(P, ctx, T, *L, log);
        W->flush = [] { throw Error(PTOWSP_ERR_PLAN, "internal: flush in a static workload"); };
        L->makespan = W->node(*plan.body, 0);
        W->close_wave();
        L->key = log;
        L->key.push_back(stride_sig);
        L->full_write.assign(T.size(), 0);
        for (size_t tid = 0; tid < T.size(); ++tid)
            L->full_write[tid] = W->fully_written(tid) ? 1 : 0;
        // a tensor that the waves overwrite entirely before any task reads it (an intermediate, like the
        // indexer's scores) need not be staged in either
        std::vector<size_t> last_w(T.size(), 0), first_r(T.size(), SIZE_MAX);
        std::vector<uint8_t> any_w(T.size(), 0);
        for (size_t wi = 0; wi < L->waves.size(); ++wi)
            for (const auto& b : L->waves[wi].batches) {
                const KernelImpl& ki = P.impls[b.kernel];
                const Node& n = *b.node;
                for (int ti = 0; ti < plan.kernels[b.kernel].num_tensor_params; ++ti) {
                    const uint32_t tid = n.tensor_args[n.param_to_arg[ti]].tensor;
                    if (ki.param_write[ti]) {
                        any_w[tid] = 1;
                        last_w[tid] = std::max(last_w[tid], wi);
                    }
                    if (ki.param_read[ti]) first_r[tid] = std::min(first_r[tid], wi);
                }
                if (b.sel) first_r[b.sel_tensor] = std::min(first_r[b.sel_tensor], wi);
            }
        L->write_first.assign(T.size(), 0);
        for (size_t tid = 0; tid < T.size(); ++tid)
            L->write_first[tid] = L->full_write[tid] && any_w[tid] && last_w[tid] < first_r[tid] ? 1 : 0;
        P.timing.walks = 1;
        if (!dry) plan_expand(P, *L, W->loops);
    }

    if (dry) {
        if (!L) {  // data-dependent workload: walk reading host memory only
            fresh = std::make_unique<LaunchProgram>();
            L = fresh.get();
            W = std::make_unique<Walker>(P, ctx, T, *L, log);
            W->flush = [] {};
            W->dry = true;
            P.timing.walks = 1;
            L->makespan = W->node(*plan.body, 0);
            W->close_wave();
            L->full_write.assign(T.size(), 0);
        }
        for (size_t tid = 0; tid < T.size(); ++tid) {
            const TensorBinding& b = T[tid];
            const bool skip = !L->full_write.empty() && L->full_write[tid] &&
                              (!b.read || (!L->write_first.empty() && L->write_first[tid]));
            if ((b.read || b.written) && !skip) P.timing.h2d_bytes += b.bytes;
            if (b.written) P.timing.d2h_bytes += b.bytes;
        }
        P.timing.tasks = L->tasks;
        for (auto& w : L->waves) {
            P.timing.waves += w.batches.empty() ? 0 : 1;
            P.timing.launches += w.batches.size();
        }
        PipePlan pp;  // would a run with these host buffers overlap its copies (kernels with a layout check on their
                      // first launch -- tcgen05 matmul, indexer scoring -- pipeline from their second run)?
        if (P.cacheable && plan_pipeline(P, *L, T, true, pp)) P.timing.chunks = static_cast<uint64_t>(pp.C);
        if (plan.body && plan.body->kind == Node::Kind::Pipeline)  // what a run would do
            P.csp_mode = L->csp && P.opt_csp_device ? std::string("device_processes")
                         : "waves: " + (!P.opt_csp_device ? std::string("csp_device option is 0")
                                        : !P.cacheable   ? std::string("data-dependent control flow")
                                                         : L->csp_note);
        return L->makespan;
    }

    // ---- overlapped copy / compute for host-staged single-batch workloads ----
    bool pipelined = false;
    if (L && !all_device && !(L->csp && P.opt_csp_device)) {
        if (replay || P.cacheable) {
            if (!replay) {
                // records must be on the device before any chunk launches
                size_t need = 0;
                for (auto& w : L->waves)
                    for (auto& b : w.batches) need += b.rec.size();
                if (need > L->rec_cap) {
                    PW_CUDA(cudaMalloc(&L->rec_dev, need * sizeof(int64_t)));
                    L->rec_cap = need;
                }
                for (auto& w : L->waves)
                    for (auto& b : w.batches) {
                        b.dev_off = L->rec_elems;
                        if (!b.rec.empty())
                            PW_CUDA(cudaMemcpyAsync(L->rec_dev + b.dev_off, b.rec.data(), b.rec.size() * sizeof(int64_t),
                                                    cudaMemcpyHostToDevice, P.stream));
                        L->rec_elems += b.rec.size();
                    }
                launched_waves = L->waves.size();  // records uploaded: the generic path must not upload again
            }
            pipelined = run_pipelined(P, *L, T, launches);
            if (!pipelined && !replay) {
                // not pipelined after all: launch what was uploaded the ordinary way below
                replay = true;
            }
        }
    }

    // ---- stage host tensors into HBM ----
    for (size_t tid = 0; tid < T.size() && !pipelined; ++tid) {
        TensorBinding& b = T[tid];
        if (b.on_device || b.bytes == 0) continue;
        // Host tensors a task touches are staged in -- outputs too, unless the
        // task loop provably overwrites every element, in waves before any
        // task reads it, so that elements no task writes come back unchanged.
        const bool skip = L && !L->full_write.empty() && L->full_write[tid] &&
                          (!b.read || (!L->write_first.empty() && L->write_first[tid]));
        if ((b.read || b.written) && !skip) {
            PW_CUDA(cudaMemcpyAsync(b.dev, b.user_ptr, b.bytes, cudaMemcpyHostToDevice, P.stream));
            P.timing.h2d_bytes += b.bytes;
        }
    }

    // the run's GPU time (`gpu_ms`) is only read back by a synchronous run
    if (!pipelined && !async_run) PW_CUDA(cudaEventRecord(P.ev0, P.stream));
    bool csp_ran = false;
    if (!pipelined && L && L->csp && P.opt_csp_device) {
        csp_ran = launch_csp(P, *L, T, launches);
        if (!csp_ran) {
            L->csp_note = "the processes cannot all be resident on the GPU at once";
            L->csp.reset();  // later replays run the waves, whose records the fallback below uploads
            if (replay) {
                // a replay of a device-process program: its waves' records were never uploaded
                throw Error(PTOWSP_ERR_CUDA, "CSP pipeline: device processes no longer fit; recompile the program");
            }
        }
    }
    if (pipelined || csp_ran) {
        // kernels and copies were enqueued by run_pipelined, or the pipeline ran as device processes
    } else if (replay) {
        for (size_t wi = 0; wi < L->waves.size(); ++wi)
            for (auto& b : L->waves[wi].batches) launch_batch(P, b, *b.node, T, L->rec_dev, launches);
    } else if (P.cacheable) {
        upload_and_launch(L->waves.size());
    } else {
        // data-dependent control flow: walk while launching (slot loads of device data flush)
        fresh = std::make_unique<LaunchProgram>();
        L = fresh.get();
        W = std::make_unique<Walker>(P, ctx, T, *L, log);
        P.timing.walks = 1;
        W->flush = [&]() {
            W->close_wave();
            upload_and_launch(L->waves.size());
            PW_CUDA(cudaStreamSynchronize(P.stream));
        };
        L->makespan = W->node(*plan.body, 0);
        W->close_wave();
        upload_and_launch(L->waves.size());
    }
    if (!pipelined && !async_run) PW_CUDA(cudaEventRecord(P.ev1, P.stream));

    // ---- bring written host tensors back ----
    for (size_t tid = 0; tid < T.size() && !pipelined; ++tid) {
        TensorBinding& b = T[tid];
        if (b.on_device || !b.written || b.bytes == 0) continue;
        PW_CUDA(cudaMemcpyAsync(b.user_ptr, b.dev, b.bytes, cudaMemcpyDeviceToHost, P.stream));
        P.timing.d2h_bytes += b.bytes;
    }
    P.timing.launches = launches;
    P.timing.tasks = L->tasks;
    P.csp_mode = plan.body && plan.body->kind == Node::Kind::Pipeline
                     ? (csp_ran ? std::string("device_processes")
                                : "waves: " + (!P.opt_csp_device ? std::string("csp_device option is 0")
                                               : !P.cacheable   ? std::string("data-dependent control flow")
                                               : L->csp_note.empty() ? std::string("not analysed") : L->csp_note))
                     : std::string();
    for (auto& w : L->waves) P.timing.waves += w.batches.empty() ? 0 : 1;
    const uint64_t makespan = L->makespan;
    int err_host = 0;
    if (!async_run) {
        // the status word accumulates over asynchronous runs; read, then clear it
        PW_CUDA(cudaMemcpyAsync(&err_host, P.err_dev, sizeof(int), cudaMemcpyDeviceToHost, P.stream));
        PW_CUDA(cudaMemsetAsync(P.err_dev, 0, sizeof(int), P.stream));
        PW_CUDA(cudaStreamSynchronize(P.stream));
        float ms = 0.f;
        cudaEventElapsedTime(&ms, P.ev0, P.ev1);
        P.timing.gpu_ms = ms;
    } else {
        P.timing.gpu_ms = -1.0;  // asynchronous run: not known yet
    }
    if (fresh) {
        if (P.cacheable && P.opt_cache) {
            if (async_run) PW_CUDA(cudaStreamSynchronize(P.stream));  // host records must outlive their copies
            for (auto& w : fresh->waves)
                for (auto& b : w.batches) std::vector<int64_t>().swap(b.rec);  // records live on the device now
            if (P.cached) PW_CUDA(cudaStreamSynchronize(P.stream));
            P.cached = std::move(fresh);
        } else {
            PW_CUDA(cudaStreamSynchronize(P.stream));
            fresh.reset();
        }
    }
    P.timing.total_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t_start).count();
    if (err_host) {
        throw Error(PTOWSP_ERR_DEVICE, std::string("device status ") + std::to_string(err_host) +
                                           ((err_host & dev::kErrBounds) ? " (index out of bounds)" : "") +
                                           ((err_host & dev::kErrTimeout) ? " (wait timed out)" : "") +
                                           ((err_host & dev::kErrShape) ? " (size beyond kernel limit)" : ""));
    }
    return makespan;
}

std::string kernel_times(Program& P) {
    PW_CUDA(cudaSetDevice(P.device));
    if (P.kev_totals.size() < P.plan.kernels.size()) P.kev_totals.resize(P.plan.kernels.size(), {0, 0.0});
    for (auto& ke : P.kev_pending) {
        PW_CUDA(cudaEventSynchronize(ke.end));
        float ms = 0.f;
        PW_CUDA(cudaEventElapsedTime(&ms, ke.start, ke.end));
        auto& t = P.kev_totals[static_cast<size_t>(ke.kernel)];
        t.first += 1;
        t.second += ms;
        P.kev_free.push_back(ke.start);
        P.kev_free.push_back(ke.end);
    }
    P.kev_pending.clear();
    std::string out = "{";
    for (size_t k = 0; k < P.plan.kernels.size(); ++k) {
        if (k) out += ",";
        char buf[160];
        std::snprintf(buf, sizeof buf, "\"launches\":%llu,\"ms\":%.6f}", static_cast<unsigned long long>(P.kev_totals[k].first),
                      P.kev_totals[k].second);
        out += "\"" + P.plan.kernels[k].name + "\":{" + buf;
    }
    return out + "}";
}

void reset_kernel_times(Program& P) {
    // unread events are dropped; they go back to the pool once their work is done
    for (auto& ke : P.kev_pending) {
        cudaEventSynchronize(ke.end);
        P.kev_free.push_back(ke.start);
        P.kev_free.push_back(ke.end);
    }
    P.kev_pending.clear();
    P.kev_totals.assign(P.plan.kernels.size(), {0, 0.0});
}

uint64_t run_single_task(Program& P, const std::string& kernel, const KernelTaskDesc* task) {
    int ki_idx = P.plan.kernel_index(kernel);
    if (ki_idx < 0) throw Error(PTOWSP_ERR_ARG, "unknown kernel " + kernel);
    if (!task) throw Error(PTOWSP_ERR_ARG, "KernelTaskDesc is null");
    const KernelDef& kd = P.plan.kernels[ki_idx];
    if (static_cast<int>(task->num_tensors) != kd.num_tensor_params)
        throw Error(PTOWSP_ERR_ARG, "tensor count does not match kernel " + kernel);
    PW_CUDA(cudaSetDevice(P.device));
    ensure_device_state(P);
    // A one-task plan node: each param views its own base pointer (offset 0).
    Node n;
    n.kind = Node::Kind::Task;
    n.kernel = kernel;
    n.kernel_index = ki_idx;
    const int naxis = static_cast<int>(task->num_axis_args) - 2 * kd.num_tensor_params;
    for (int i = 0; i < std::max(naxis, 0); ++i) n.axis_args.push_back(ArgSpec{ArgSpec::Kind::U64, "", task->args[i]});
    std::vector<TensorBinding> T(kd.num_tensor_params);
    Batch b;
    b.kernel = ki_idx;
    b.ntasks = 1;
    b.stride = kd.num_tensor_params + std::max(naxis, 0) + kd.num_scalar_params;
    for (int ti = 0; ti < kd.num_tensor_params; ++ti) {
        TensorArg ta;
        ta.tensor = static_cast<uint32_t>(ti);
        ta.base_rank = 2;
        ta.view_rank = 2;
        n.tensor_args.push_back(ta);
        n.param_to_arg.push_back(ti);
        T[ti].dev = static_cast<char*>(task->tensor_ptrs[ti]);
        T[ti].strides = {static_cast<int64_t>(task->tensor_strides[2 * ti]), static_cast<int64_t>(task->tensor_strides[2 * ti + 1])};
        T[ti].span = INT64_MAX / 16;
        b.rec.push_back(0);
    }
    for (int i = 0; i < std::max(naxis, 0); ++i) b.rec.push_back(static_cast<int64_t>(task->args[i]));
    for (int i = 0; i < kd.num_scalar_params; ++i) b.rec.push_back(static_cast<int64_t>(task->args[task->num_axis_args + i]));
    int64_t* rec_dev = nullptr;
    PW_CUDA(cudaMalloc(&rec_dev, b.rec.size() * sizeof(int64_t)));
    PW_CUDA(cudaMemcpyAsync(rec_dev, b.rec.data(), b.rec.size() * sizeof(int64_t), cudaMemcpyHostToDevice, P.stream));
    uint64_t launches = 0;
    launch_batch(P, b, n, T, rec_dev, launches);
    int err_host = 0;
    PW_CUDA(cudaMemcpyAsync(&err_host, P.err_dev, sizeof(int), cudaMemcpyDeviceToHost, P.stream));
    PW_CUDA(cudaMemsetAsync(P.err_dev, 0, sizeof(int), P.stream));
    PW_CUDA(cudaStreamSynchronize(P.stream));
    cudaFree(rec_dev);
    if (err_host) throw Error(PTOWSP_ERR_DEVICE, "device status " + std::to_string(err_host));
    return P.impls[ki_idx].cycles;
}

}  // namespace ptowsp
