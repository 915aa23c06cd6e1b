// Plan compilation: every kernel definition is matched to a CUDA
// implementation (hand-written kernel, built-in, or the generic tile program)
// and given its reference cycle-model charge.  There is no CPU fallback: a
// kernel the GPU cannot run is a compile error, like an unsupported target in
// compile_codegen (src/python/pto_codegen.cpp:3433).
#include <algorithm>
#include <cstring>
#include <functional>
#include <set>
#include <sstream>

#include "runtime.hpp"

namespace ptowsp {

const char* impl_name(ImplKind k) {
    switch (k) {
        case ImplKind::RmsNorm: return "rmsnorm_rows";
        case ImplKind::Softmax: return "softmax_rows";
        case ImplKind::TileProgram: return "tile_program";
        case ImplKind::Matmul: return "matmul_tcgen05";
        case ImplKind::MatmulAcc: return "matmul_tcgen05_acc";
        case ImplKind::MatmulEpilogue: return "matmul_tcgen05+row_program";
        case ImplKind::PagedDecode: return "paged_decode_gqa";
        case ImplKind::IndexerScore: return "lightning_indexer_score";
        case ImplKind::TopK: return "topk_select";
        case ImplKind::Staged: return "staged_matmul+row_programs";
        case ImplKind::Attention: return "attention_tcgen05";
    }
    return "?";
}

namespace {

bool is_float(DType d) { return d == DType::F32 || d == DType::F16 || d == DType::BF16 || d == DType::F64; }

int word_of(DType d) {
    if (is_float(d)) return dev::W_F32;
    if (d == DType::U8 || d == DType::U16 || d == DType::U32 || d == DType::U64) return dev::W_U32;
    return dev::W_I32;
}

// Which param tiles the reference pre-loads: params read by any op other than
// Matmul/Load, excluding the Store destination (collect_param_tiles_to_load,
// src/python/pto_codegen.cpp:448-468).
std::set<int> preload_set(const KernelDef& kd) {
    std::set<int> used;
    for (const auto& op : kd.ops) {
        if (op.kind == "Matmul" || op.kind == "Load") continue;
        for (size_t i = 0; i < op.operands.size(); ++i) {
            int oid = op.operands[i];
            auto it = kd.values.find(oid);
            if (it == kd.values.end() || !it->second.is_tile()) continue;
            if (!kd.param_by_id(oid)) continue;
            if (op.kind == "Store" && i == 0) continue;
            used.insert(oid);
        }
    }
    return used;
}

struct ScalarConst {
    bool is_param = false;
    int scalar_index = -1;
    DType dtype = DType::F32;
    double value = 0.0;
};

// ---------------------------------------------------------------------------
// One pass over the ops that both charges the reference cycle model
// (include/pto/wsp/codegen/abi/ptoisa_bridge.hpp:67-303) and, when `tp` is
// given, records the GPU tile program.  Ops the reference emitter skips are
// skipped here too (no code, and no cycles except the "unhandled op" charge).
// ---------------------------------------------------------------------------
struct KernelWalker {
    const KernelDef& kd;
    dev::TileProgram* tp;
    uint64_t cycles = 0;
    std::map<int, int> slot_of;  // value id -> slot
    std::set<int> local;         // op-result tiles + preloaded params
    std::map<int, ScalarConst> scalars;
    std::map<int, std::pair<int, int>> store_dims;
    std::vector<uint8_t> written, read;
    std::string error;
    int words = 0;

    explicit KernelWalker(const KernelDef& k, dev::TileProgram* t) : kd(k), tp(t) {
        written.assign(kd.num_tensor_params, 0);
        read.assign(kd.num_tensor_params, 0);
        if (tp) std::memset(tp, 0, sizeof(*tp));
    }

    std::pair<int, int> vdims(int vid) const {
        auto it = store_dims.find(vid);
        if (it != store_dims.end()) return it->second;
        const auto& v = kd.values.at(vid);
        return {v.rows, v.cols};
    }

    int new_slot(int rows, int cols, DType dt) {
        if (!tp) return -1;
        if (tp->nslots >= dev::kTPMaxSlots) {
            error = "too many tiles for the tile program";
            return -1;
        }
        dev::TPSlot s{};
        s.off = words;
        s.rows = rows;
        s.cols = cols;
        s.pitch = cols;
        s.word = word_of(dt);
        words += rows * cols;
        tp->slots[tp->nslots] = s;
        return tp->nslots++;
    }

    void emit(const dev::TPInstr& in) {
        if (!tp) return;
        if (tp->ninstr >= dev::kTPMaxInstr) {
            error = "too many ops for the tile program";
            return;
        }
        tp->ins[tp->ninstr++] = in;
    }

    int slot(int vid) {
        auto it = slot_of.find(vid);
        return it == slot_of.end() ? -1 : it->second;
    }

    void run() {
        // scalar params / constants usable by the scalar fast path (pto_codegen.cpp:563-610)
        for (const auto& p : kd.params) {
            if (p.v.is_tile()) continue;
            if (p.v.dtype == DType::F32 || p.v.dtype == DType::I32 || p.v.dtype == DType::I64 || p.v.dtype == DType::Bool) {
                ScalarConst sc;
                sc.is_param = true;
                sc.scalar_index = p.scalar_index;
                sc.dtype = p.v.dtype;
                scalars[p.id] = sc;
                if (tp) tp->scalar_types[p.scalar_index] = p.v.dtype == DType::F32 ? 0 : p.v.dtype == DType::I32 ? 1 : p.v.dtype == DType::I64 ? 2 : 3;
            }
        }
        for (const auto& op : kd.ops) {
            if (op.kind != "Constant" || op.result < 0) continue;
            auto it = kd.values.find(op.result);
            if (it == kd.values.end() || it->second.is_tile()) continue;
            auto* v = op.attrs.get("value");
            if (!v) continue;
            ScalarConst sc;
            sc.dtype = it->second.dtype;
            sc.value = v->as_f64();
            scalars[op.result] = sc;
        }
        for (const auto& op : kd.ops) {
            if (op.kind != "Store" || op.operands.size() < 2) continue;
            const KernelParam* dst = kd.param_by_id(op.operands[0]);
            if (dst && dst->v.is_tile()) store_dims[op.operands[1]] = {dst->v.rows, dst->v.cols};
        }
        // local tiles
        for (const auto& op : kd.ops) {
            if (op.result < 0 || kd.param_by_id(op.result)) continue;
            auto it = kd.values.find(op.result);
            if (it == kd.values.end() || !it->second.is_tile()) continue;
            local.insert(op.result);
        }
        auto pre = preload_set(kd);
        for (int pid : pre) local.insert(pid);
        // allocate slots for local tiles
        for (int vid : local) {
            const auto& v = kd.values.at(vid);
            slot_of[vid] = new_slot(v.rows, v.cols, v.dtype);
        }
        for (int pid : pre) {
            const KernelParam* p = kd.param_by_id(pid);
            cycles += static_cast<uint64_t>(p->v.rows) * p->v.cols;
            read[p->tensor_index] = 1;
            dev::TPInstr in{};
            in.op = dev::TP_LOAD;
            in.dst = slot(pid);
            in.param = p->tensor_index;
            in.rows = p->v.rows;
            in.cols = p->v.cols;
            emit(in);
        }
        for (const auto& op : kd.ops) step(op);
        if (tp) tp->smem_words = words;
    }

    void unhandled(const OpInfo& op) {
        if (op.result >= 0) {
            auto it = kd.values.find(op.result);
            if (it != kd.values.end() && it->second.is_tile())
                cycles += static_cast<uint64_t>(it->second.rows) * it->second.cols;
        }
    }

    void step(const OpInfo& op) {
        const std::string& k = op.kind;
        const int rid = op.result;
        const auto& ops = op.operands;
        if (k == "Load") {
            if (rid < 0 || ops.empty() || !local.count(rid)) return;
            const KernelParam* src = kd.param_by_id(ops[0]);
            if (!src || !src->v.is_tile()) return;
            auto [r, c] = vdims(rid);
            cycles += static_cast<uint64_t>(r) * c;
            read[src->tensor_index] = 1;
            dev::TPInstr in{};
            in.op = dev::TP_LOAD;
            in.dst = slot(rid);
            in.param = src->tensor_index;
            in.rows = src->v.rows;
            in.cols = src->v.cols;
            emit(in);
            return;
        }
        if (k == "Matmul") {
            if (rid < 0 || ops.size() < 2 || !local.count(rid)) return;
            auto info = [&](int oid, int& r, int& c, DType& dt, bool& is_param) -> bool {
                if (const KernelParam* p = kd.param_by_id(oid)) {
                    if (!p->v.is_tile()) return false;
                    r = p->v.rows, c = p->v.cols, dt = p->v.dtype, is_param = true;
                    return true;
                }
                if (local.count(oid)) {
                    const auto& v = kd.values.at(oid);
                    r = v.rows, c = v.cols, dt = v.dtype, is_param = false;
                    return true;
                }
                return false;
            };
            int ar, ac, br, bc;
            DType adt, bdt;
            bool ap, bp;
            if (!info(ops[0], ar, ac, adt, ap) || !info(ops[1], br, bc, bdt, bp)) return;
            if (ac != br) return;
            DType rdt = kd.values.at(rid).dtype;
            bool ok = (adt == DType::F32 && bdt == DType::F32 && rdt == DType::F32) ||
                      (adt == DType::F16 && bdt == DType::F16 && rdt == DType::F32);
            if (!ok) return;
            cycles += static_cast<uint64_t>(ar) * ac;                 // TLOAD/TMOV TileLeft
            cycles += static_cast<uint64_t>(br) * bc;                 // TLOAD/TMOV TileRight
            cycles += static_cast<uint64_t>(ar) * ac * bc;            // TMATMUL
            int sa = -1, sb = -1;
            if (ap) {
                const KernelParam* p = kd.param_by_id(ops[0]);
                read[p->tensor_index] = 1;
                sa = new_slot(ar, ac, adt);
                dev::TPInstr in{};
                in.op = dev::TP_LOAD;
                in.dst = sa;
                in.param = p->tensor_index;
                in.rows = ar;
                in.cols = ac;
                emit(in);
            } else {
                sa = slot(ops[0]);
            }
            if (bp) {
                const KernelParam* p = kd.param_by_id(ops[1]);
                read[p->tensor_index] = 1;
                sb = new_slot(br, bc, bdt);
                dev::TPInstr in{};
                in.op = dev::TP_LOAD;
                in.dst = sb;
                in.param = p->tensor_index;
                in.rows = br;
                in.cols = bc;
                emit(in);
            } else {
                sb = slot(ops[1]);
            }
            dev::TPInstr in{};
            in.op = dev::TP_MATMUL;
            in.dst = slot(rid);
            in.a = sa;
            in.b = sb;
            in.rows = ar;
            in.cols = bc;
            in.k = ac;
            emit(in);
            // acc -> vec TMOV when a non-matmul, non-store op consumes the accumulator
            for (const auto& o2 : kd.ops) {
                if (o2.kind == "Matmul" || o2.kind == "Store") continue;
                if (std::find(o2.operands.begin(), o2.operands.end(), rid) != o2.operands.end()) {
                    auto [r, c] = vdims(rid);
                    cycles += static_cast<uint64_t>(r) * c;
                    break;
                }
            }
            return;
        }
        if (k == "Store") {
            if (ops.size() < 2) return;
            const KernelParam* dst = kd.param_by_id(ops[0]);
            if (!dst || !dst->v.is_tile()) return;
            int src = ops[1];
            if (!local.count(src)) return;
            DType sdt = kd.values.at(src).dtype;
            if (dst->v.dtype != sdt && !(dst->v.dtype == DType::F16 && sdt == DType::F32)) return;
            uint64_t rc = static_cast<uint64_t>(dst->v.rows) * dst->v.cols;
            if (dst->v.dtype != sdt) cycles += rc;  // TCVT
            cycles += rc;                            // TSTORE
            written[dst->tensor_index] = 1;
            dev::TPInstr in{};
            in.op = dev::TP_STORE;
            in.a = slot(src);
            in.param = dst->tensor_index;
            in.rows = dst->v.rows;
            in.cols = dst->v.cols;
            emit(in);
            return;
        }
        if (k == "Add" || k == "Sub" || k == "Mul" || k == "Div" || k == "Max" || k == "Min") {
            if (rid < 0 || ops.size() != 2 || !local.count(rid)) return;
            int sub = k == "Add" ? dev::BIN_ADD : k == "Sub" ? dev::BIN_SUB : k == "Mul" ? dev::BIN_MUL
                    : k == "Div" ? dev::BIN_DIV : k == "Max" ? dev::BIN_MAX : dev::BIN_MIN;
            bool as = scalars.count(ops[0]) != 0, bs = scalars.count(ops[1]) != 0;
            auto [r, c] = vdims(rid);
            if (as != bs) {
                int tid = as ? ops[1] : ops[0];
                int sid = as ? ops[0] : ops[1];
                if (!local.count(tid)) return;
                if (k == "Sub" && as) return;  // scalar - tile not supported (pto_codegen.cpp:1040)
                cycles += static_cast<uint64_t>(r) * c;
                const ScalarConst& sc = scalars.at(sid);
                dev::TPInstr in{};
                in.op = dev::TP_BINS;
                in.sub = sub;
                in.dst = slot(rid);
                in.a = slot(tid);
                in.scalar_src = sc.is_param ? sc.scalar_index : -1;
                in.scalar_first = (k == "Div" && as) ? 1 : 0;
                in.fval = static_cast<float>(sc.value);
                in.ival = static_cast<int>(sc.value);
                emit(in);
                return;
            }
            if (!local.count(ops[0]) || !local.count(ops[1])) return;
            const auto& va = kd.values.at(ops[0]);
            const auto& vb = kd.values.at(ops[1]);
            const auto& vr = kd.values.at(rid);
            int mode = -1;
            if (va.rows == vr.rows && va.cols == vr.cols && vb.rows == vr.rows && vb.cols == vr.cols) mode = dev::MODE_FULL;
            else if (va.rows == vr.rows && va.cols == vr.cols &&
                     ((vb.rows == vr.rows && vb.cols == 1) || (vb.rows == 1 && vb.cols == vr.rows)))
                mode = dev::MODE_ROW;
            else if ((k == "Sub" || k == "Mul" || k == "Div") && va.rows == vr.rows && va.cols == vr.cols &&
                     ((vb.rows == 1 && vb.cols == vr.cols) || (vb.rows == vr.cols && vb.cols == 1)))
                mode = dev::MODE_COL;
            if (mode < 0) return;  // broadcast pattern unsupported: no code, no cycles
            cycles += static_cast<uint64_t>(r) * c;
            dev::TPInstr in{};
            in.op = dev::TP_BIN;
            in.sub = sub;
            in.mode = mode;
            in.dst = slot(rid);
            in.a = slot(ops[0]);
            in.b = slot(ops[1]);
            emit(in);
            return;
        }
        if (k == "Exp" || k == "Rsqrt") {
            if (rid < 0 || ops.size() != 1 || !local.count(rid) || !local.count(ops[0])) return;
            auto [r, c] = vdims(rid);
            cycles += static_cast<uint64_t>(r) * c;
            dev::TPInstr in{};
            in.op = k == "Exp" ? dev::TP_EXP : dev::TP_RSQRT;
            in.dst = slot(rid);
            in.a = slot(ops[0]);
            emit(in);
            return;
        }
        if (k == "IotaU32") {
            if (rid < 0 || !local.count(rid)) return;
            const auto& v = kd.values.at(rid);
            if (v.rows != 1) return;
            dev::TPInstr in{};
            in.op = dev::TP_IOTA;
            in.dst = slot(rid);
            emit(in);
            return;
        }
        if (k == "TSort32") {
            if (rid < 0 || ops.size() != 2 || !local.count(rid) || !local.count(ops[0]) || !local.count(ops[1])) return;
            int sr, sc;
            if (const KernelParam* p = kd.param_by_id(ops[0])) sr = p->v.rows, sc = p->v.cols;
            else std::tie(sr, sc) = vdims(ops[0]);
            cycles += 5ull * static_cast<uint64_t>(sr) * sc;
            dev::TPInstr in{};
            in.op = dev::TP_TSORT32;
            in.dst = slot(rid);
            in.a = slot(ops[0]);
            in.b = slot(ops[1]);
            in.k = sr * sc;
            emit(in);
            return;
        }
        if (k == "ExtractTopkIndices") {
            if (rid < 0 || ops.size() != 1 || !local.count(rid) || !local.count(ops[0])) return;
            int kk = 0;
            if (auto* a = op.attrs.get("k")) kk = static_cast<int>(a->as_i64());
            if (kk <= 0) kk = kd.values.at(rid).cols;
            dev::TPInstr in{};
            in.op = dev::TP_EXTRACT;
            in.dst = slot(rid);
            in.a = slot(ops[0]);
            in.k = kk;
            emit(in);
            return;
        }
        if (k == "RowSum" || k == "RowMax" || k == "RowMean") {
            if (rid < 0 || ops.size() != 1 || !local.count(rid) || !local.count(ops[0])) return;
            auto [r, c] = vdims(rid);
            cycles += static_cast<uint64_t>(r) * c * (k == "RowMean" ? 2u : 1u);
            dev::TPInstr in{};
            in.op = k == "RowSum" ? dev::TP_ROWSUM : k == "RowMax" ? dev::TP_ROWMAX : dev::TP_ROWMEAN;
            in.dst = slot(rid);
            in.a = slot(ops[0]);
            in.k = kd.values.at(ops[0]).cols;
            emit(in);
            return;
        }
        unhandled(op);
    }
};

bool match_ops(const KernelDef& kd, const std::vector<std::string>& kinds) {
    if (kd.ops.size() != kinds.size()) return false;
    for (size_t i = 0; i < kinds.size(); ++i)
        if (kd.ops[i].kind != kinds[i]) return false;
    return true;
}

bool is_tile_param(const KernelDef& kd, int id, DType dt) {
    const KernelParam* p = kd.param_by_id(id);
    return p && p->v.is_tile() && p->v.dtype == dt;
}

// RMSNorm: Mul(x,x) RowMean Rsqrt Mul(x,inv) Store  (examples/e2e_rmsnorm/pto_wsp_impl.py:43-52)
bool is_rmsnorm(const KernelDef& kd) {
    if (!match_ops(kd, {"Mul", "RowMean", "Rsqrt", "Mul", "Store"})) return false;
    const auto& o = kd.ops;
    int x = o[0].operands.size() == 2 ? o[0].operands[0] : -1;
    if (x < 0 || o[0].operands[1] != x || !is_tile_param(kd, x, DType::F32)) return false;
    if (o[1].operands != std::vector<int>{o[0].result}) return false;
    if (o[2].operands != std::vector<int>{o[1].result}) return false;
    if (o[3].operands != std::vector<int>{x, o[2].result}) return false;
    if (o[4].operands.size() != 2 || o[4].operands[1] != o[3].result || !is_tile_param(kd, o[4].operands[0], DType::F32))
        return false;
    const auto& vx = kd.values.at(x);
    const auto& vo = kd.param_by_id(o[4].operands[0])->v;
    const auto& vm = kd.values.at(o[1].result);
    return vx.rows == vo.rows && vx.cols == vo.cols && vm.rows == vx.rows && vm.cols == 1 &&
           kd.values.at(o[3].result).dtype == DType::F32 && kd.num_tensor_params == 2;
}

// Softmax: RowMax Sub Exp RowSum Div Store
bool is_softmax(const KernelDef& kd) {
    if (!match_ops(kd, {"RowMax", "Sub", "Exp", "RowSum", "Div", "Store"})) return false;
    const auto& o = kd.ops;
    int x = o[0].operands.size() == 1 ? o[0].operands[0] : -1;
    if (x < 0 || !is_tile_param(kd, x, DType::F32)) return false;
    if (o[1].operands != std::vector<int>{x, o[0].result}) return false;
    if (o[2].operands != std::vector<int>{o[1].result}) return false;
    if (o[3].operands != std::vector<int>{o[2].result}) return false;
    if (o[4].operands != std::vector<int>{o[2].result, o[3].result}) return false;
    if (o[5].operands.size() != 2 || o[5].operands[1] != o[4].result || !is_tile_param(kd, o[5].operands[0], DType::F32))
        return false;
    const auto& vx = kd.values.at(x);
    const auto& vo = kd.param_by_id(o[5].operands[0])->v;
    return vx.rows == vo.rows && vx.cols == vo.cols && kd.values.at(o[0].result).cols == 1 &&
           kd.values.at(o[4].result).dtype == DType::F32 && kd.num_tensor_params == 2;
}

// Matmul: C = A.B (f16 x f16 -> f32), optionally C += A.B (examples/bgemm/pto_wsp_impl.py:56-76).
int matmul_form(const KernelDef& kd) {
    const auto& o = kd.ops;
    if (kd.num_tensor_params != 3 || kd.num_scalar_params != 0) return 0;
    auto check_ab = [&](const OpInfo& mm) {
        return mm.operands.size() == 2 && is_tile_param(kd, mm.operands[0], DType::F16) &&
               is_tile_param(kd, mm.operands[1], DType::F16) && kd.values.at(mm.result).dtype == DType::F32 &&
               kd.param_by_id(mm.operands[0])->v.cols == kd.param_by_id(mm.operands[1])->v.rows;
    };
    if (match_ops(kd, {"Matmul", "Store"})) {
        if (!check_ab(o[0])) return 0;
        if (o[1].operands.size() != 2 || o[1].operands[1] != o[0].result) return 0;
        if (!is_tile_param(kd, o[1].operands[0], DType::F32)) return 0;
        const auto& vc = kd.param_by_id(o[1].operands[0])->v;
        const auto& va = kd.param_by_id(o[0].operands[0])->v;
        const auto& vb = kd.param_by_id(o[0].operands[1])->v;
        return (vc.rows == va.rows && vc.cols == vb.cols) ? 1 : 0;
    }
    if (match_ops(kd, {"Matmul", "Add", "Store"})) {
        if (!check_ab(o[0])) return 0;
        const auto& add = o[1];
        if (add.operands.size() != 2) return 0;
        int c = add.operands[0] == o[0].result ? add.operands[1] : add.operands[0];
        if (std::find(add.operands.begin(), add.operands.end(), o[0].result) == add.operands.end()) return 0;
        if (!is_tile_param(kd, c, DType::F32)) return 0;
        if (o[2].operands != std::vector<int>{c, add.result}) return 0;
        const auto& vc = kd.param_by_id(c)->v;
        const auto& va = kd.param_by_id(o[0].operands[0])->v;
        const auto& vb = kd.param_by_id(o[0].operands[1])->v;
        return (vc.rows == va.rows && vc.cols == vb.cols) ? 2 : 0;
    }
    return 0;
}

const KernelParam& tparam(const KernelDef& kd, int ti) {
    for (const auto& p : kd.params)
        if (p.tensor_index == ti) return p;
    throw Error(PTOWSP_ERR_PLAN, "kernel " + kd.name + ": missing tensor param");
}

void setup_builtin(const KernelDef& kd, KernelImpl& ki) {
    const std::string& b = kd.builtin;
    auto need = [&](int nt, int ns) {
        if (kd.num_tensor_params != nt || kd.num_scalar_params != ns)
            throw Error(PTOWSP_ERR_PLAN, "built-in " + b + " expects " + std::to_string(nt) + " tile params and " +
                                             std::to_string(ns) + " scalar params (kernel " + kd.name + ")");
    };
    ki.param_read.assign(kd.num_tensor_params, 1);
    ki.param_write.assign(kd.num_tensor_params, 0);
    if (b == "paged_decode_gqa") {
        need(6, 2);
        ki.kind = ImplKind::PagedDecode;
        const auto& q = tparam(kd, 0).v;
        const auto& pt = tparam(kd, 3).v;
        if (q.dtype != DType::F16 || tparam(kd, 1).v.dtype != DType::F16 || tparam(kd, 2).v.dtype != DType::F16 ||
            pt.dtype != DType::I32 || tparam(kd, 4).v.dtype != DType::I32 || tparam(kd, 5).v.dtype != DType::F16)
            throw Error(PTOWSP_ERR_PLAN, "paged_decode_gqa: dtypes must be q/k/v/out f16, page_table/kv_len i32");
        if (q.cols != 128) throw Error(PTOWSP_ERR_UNSUPPORTED, "paged_decode_gqa: head_dim must be 128");
        if (q.rows != 1 && q.rows != 2 && q.rows != 4 && q.rows != 8)
            throw Error(PTOWSP_ERR_UNSUPPORTED, "paged_decode_gqa: GQA group of 1, 2, 4 or 8 query heads");
        ki.param_write[5] = 1;
        ki.param_read[5] = 0;
        // Model charge with the static maximum length (page_table width x page size):
        // G*D + 2*L*D + G*D*L + 5*G*L + 2*G + G*L*D + G*D, see oracle/cpu_sim.py.
        const uint64_t G = q.rows, D = q.cols;
        const uint64_t L = static_cast<uint64_t>(pt.cols) * 16ull;
        ki.cycles = G * D + 2 * L * D + G * D * L + 5 * G * L + 2 * G + G * L * D + G * D;
    } else if (b == "lightning_indexer_score") {
        need(4, 0);
        ki.kind = ImplKind::IndexerScore;
        const auto& q = tparam(kd, 0).v;
        const auto& k = tparam(kd, 1).v;
        const auto& w = tparam(kd, 2).v;
        const auto& s = tparam(kd, 3).v;
        if (q.dtype != DType::F16 || k.dtype != DType::F16 || w.dtype != DType::F32 || s.dtype != DType::F32)
            throw Error(PTOWSP_ERR_PLAN, "lightning_indexer_score: q,k f16; w, scores f32");
        if (q.cols != 128 || k.cols != 128) throw Error(PTOWSP_ERR_UNSUPPORTED, "lightning_indexer_score: head_dim must be 128");
        if (w.rows * w.cols != q.rows || s.rows != w.rows || s.cols != k.rows)
            throw Error(PTOWSP_ERR_PLAN, "lightning_indexer_score: shapes q[Q*H,D] k[T,D] w[Q,H] scores[Q,T]");
        if (w.cols != 64 || w.rows != 8 || k.rows % 128 != 0)
            throw Error(PTOWSP_ERR_UNSUPPORTED, "lightning_indexer_score: 8 queries x 64 heads, keys a multiple of 128");
        ki.param_write[3] = 1;
        ki.param_read[3] = 0;
        const uint64_t QH = q.rows, D = q.cols, T = k.rows, Q = w.rows;
        ki.cycles = QH * D + T * D + QH * D * T + 2 * QH * T + Q * T;
    } else if (b == "topk_select") {
        need(2, 0);
        ki.kind = ImplKind::TopK;
        const auto& s = tparam(kd, 0).v;
        const auto& o = tparam(kd, 1).v;
        if (s.dtype != DType::F32 || o.dtype != DType::I32 || s.rows != 1 || o.rows != 1)
            throw Error(PTOWSP_ERR_PLAN, "topk_select: scores f32 [1,N] -> indices i32 [1,K]");
        if (o.cols > s.cols) throw Error(PTOWSP_ERR_PLAN, "topk_select: K > N");
        if (!dev::topk_supported(s.cols, o.cols))
            throw Error(PTOWSP_ERR_LIMIT, "topk_select: K <= 4096 and 4 N + 8 K (K rounded up to a power of two) "
                                          "+ 16 KB within 225 KB of shared memory (N <= 49152 at K = 2048)");
        ki.param_write[1] = 1;
        ki.param_read[1] = 0;
        const uint64_t N = s.cols, K = o.cols;
        ki.cycles = N + 5 * N + K;
    } else {
        throw Error(PTOWSP_ERR_UNSUPPORTED, "unknown built-in kernel '" + b + "' (kernel " + kd.name + ")");
    }
}

void collect_depths(const Plan& plan, const Node& n, std::vector<int>& depth) {
    auto see = [&](const TensorArg& ta) {
        int d = static_cast<int>(ta.index.size());
        int& cur = depth[ta.tensor];
        cur = cur < 0 ? d : std::min(cur, d);
    };
    switch (n.kind) {
        case Node::Kind::ParallelFor:
        case Node::Kind::ForEach:
        case Node::Kind::Select:
        case Node::Kind::Send:
        case Node::Kind::Consume:
            collect_depths(plan, *n.body, depth);
            break;
        case Node::Kind::Combine:
        case Node::Kind::Sequential:
        case Node::Kind::Pipeline:
            for (auto& c : n.children) collect_depths(plan, *c, depth);
            break;
        case Node::Kind::Cond:
            collect_depths(plan, *n.then_n, depth);
            collect_depths(plan, *n.else_n, depth);
            break;
        case Node::Kind::Task: {
            for (auto& ta : n.tensor_args) see(ta);
            // A tile larger than its view reaches into the neighbouring views (the reference walks such tasks in
            // program order, so the overlap is ordered): the tensor's hazard key is then the whole tensor.
            if (n.kernel_index < 0 || n.kernel_index >= static_cast<int>(plan.kernels.size())) break;
            const KernelDef& kd = plan.kernels[n.kernel_index];
            for (const auto& kp : kd.params) {
                if (kp.tensor_index < 0 || kp.tensor_index >= static_cast<int>(n.param_to_arg.size())) continue;
                const TensorArg& ta = n.tensor_args[n.param_to_arg[kp.tensor_index]];
                const auto& shape = plan.tensors[ta.tensor].shape;
                const int first = ta.base_rank - ta.view_rank;  // the view's first dimension
                int64_t vr = 1, vc = 1;
                if (ta.view_rank >= 2) {
                    vr = first < static_cast<int>(shape.size()) ? shape[first] : -1;
                    vc = first + 1 < static_cast<int>(shape.size()) ? shape[first + 1] : -1;
                } else if (ta.view_rank == 1) {
                    vc = first < static_cast<int>(shape.size()) ? shape[first] : -1;
                }
                const bool known = vr > 0 && vc > 0;
                const bool rows_over = ta.view_rank >= 2 && kp.v.rows > vr;  // a 1-D view repeats its row (s3 = 0)
                if (known && (rows_over || kp.v.cols > vc)) depth[ta.tensor] = 0;
            }
            break;
        }
        case Node::Kind::SlotLoad:
            see(n.slot_tensor);
            break;
        default:
            break;
    }
}

// ---- device-selected scalars ----

bool same_index(const std::vector<IndexExpr>& a, const std::vector<IndexExpr>& b) {
    if (a.size() != b.size()) return false;
    for (size_t i = 0; i < a.size(); ++i)
        if (a[i].is_var != b[i].is_var || a[i].var != b[i].var || a[i].c != b[i].c) return false;
    return true;
}

bool same_task_shape(const Node& a, const Node& b) {  // kernel, axis args and views equal; scalars may differ
    if (a.kernel_index != b.kernel_index || a.axis_args.size() != b.axis_args.size() ||
        a.tensor_args.size() != b.tensor_args.size() || a.scalar_args.size() != b.scalar_args.size())
        return false;
    for (size_t i = 0; i < a.axis_args.size(); ++i)
        if (a.axis_args[i].kind != b.axis_args[i].kind || a.axis_args[i].var != b.axis_args[i].var ||
            a.axis_args[i].v != b.axis_args[i].v)
            return false;
    for (size_t i = 0; i < a.tensor_args.size(); ++i) {
        const TensorArg &x = a.tensor_args[i], &y = b.tensor_args[i];
        if (x.param != y.param || x.tensor != y.tensor || x.base_rank != y.base_rank || x.view_rank != y.view_rank ||
            !same_index(x.index, y.index))
            return false;
    }
    return true;
}

bool expr_mentions(const Expr* e, Expr::Op op, bool any_value, uint64_t v) {
    if (!e) return false;
    if (e->op == op && (any_value || e->v == v)) return true;
    return expr_mentions(e->a.get(), op, any_value, v) || expr_mentions(e->b.get(), op, any_value, v) ||
           expr_mentions(e->c.get(), op, any_value, v);
}

// Builds the DevSelect of cond tree `n` over slot `slot`; false when the tree has another shape.
bool build_select(const Node& n, uint32_t slot, DevSelect& ds, int& code) {
    if (n.kind == Node::Kind::Task) {
        if (!ds.leaves.empty() && !same_task_shape(*ds.leaves[0], n)) return false;
        ds.leaves.push_back(&n);
        code = ~static_cast<int>(ds.leaves.size() - 1);
        return true;
    }
    if (n.kind != Node::Kind::Cond || !n.pred || n.pred->op != Expr::Op::Binary) return false;
    const Expr& p = *n.pred;
    static const char* cmps[] = {"<", "<=", ">", ">=", "==", "!="};
    if (std::find_if(std::begin(cmps), std::end(cmps), [&](const char* c) { return p.fn == c; }) == std::end(cmps))
        return false;
    const bool left = p.a && p.a->op == Expr::Op::Slot && p.a->v == slot;
    const bool right = p.b && p.b->op == Expr::Op::Slot && p.b->v == slot;
    if (left == right) return false;
    const Expr* other = left ? p.b.get() : p.a.get();
    const Expr* sl = left ? p.a.get() : p.b.get();
    if (sl->ty == Expr::Ty::Bool) return false;  // a slot read as bool: keep the host path
    if (expr_mentions(other, Expr::Op::Slot, true, 0) || expr_mentions(other, Expr::Op::TaskParam, true, 0))
        return false;
    const int me = static_cast<int>(ds.cmp.size());
    ds.cmp.push_back(p.fn);
    ds.slot_left.push_back(left ? 1 : 0);
    ds.other.push_back(other);
    ds.slot_expr.push_back(sl);
    ds.then_c.push_back(0);
    ds.else_c.push_back(0);
    int t = 0, e = 0;
    if (!build_select(*n.then_n, slot, ds, t) || !build_select(*n.else_n, slot, ds, e)) return false;
    ds.then_c[me] = t;
    ds.else_c[me] = e;
    code = me;
    return true;
}

// Every place slot `slot` is set or read, besides the load and tree of a candidate.
int slot_uses(const Node& n, uint32_t slot) {
    int u = 0;
    if ((n.kind == Node::Kind::SlotLoad || n.kind == Node::Kind::SlotSet) && n.slot == slot) ++u;
    if (n.kind == Node::Kind::Cond && expr_mentions(n.pred.get(), Expr::Op::Slot, false, slot)) ++u;
    if (n.body) u += slot_uses(*n.body, slot);
    for (auto& c : n.children) u += slot_uses(*c, slot);
    if (n.then_n) u += slot_uses(*n.then_n, slot);
    if (n.else_n) u += slot_uses(*n.else_n, slot);
    return u;
}

int cond_count(const Node& n) { return n.kind == Node::Kind::Cond ? 1 + cond_count(*n.then_n) + cond_count(*n.else_n) : 0; }

void find_dev_selects(Plan& plan, const std::vector<KernelImpl>& impls, Node& n) {
    if (n.kind == Node::Kind::Pipeline) return;  // process bodies keep the host walk
    if (n.kind == Node::Kind::Sequential || n.kind == Node::Kind::Combine) {
        for (size_t i = 0; i + 1 < n.children.size(); ++i) {
            Node& ld = *n.children[i];
            Node& cd = *n.children[i + 1];
            if (ld.kind != Node::Kind::SlotLoad || cd.kind != Node::Kind::Cond || cd.dev_select) continue;
            // the slot serves this tree alone: one load, and read by this tree's conds only
            if (slot_uses(*plan.body, ld.slot) != 1 + cond_count(cd)) continue;
            if (plan.schedule.dispatch_key && expr_mentions(plan.schedule.dispatch_key.get(), Expr::Op::TaskParam, true, 0))
                continue;  // a key over task params could tell the leaves apart
            auto ds = std::make_shared<DevSelect>();
            int code = 0;
            if (!build_select(cd, ld.slot, *ds, code) || ds->leaves.size() < 2) continue;
            // the leaves' kernel must read its scalars from the device records (the generic tile program)
            if (impls[ds->leaves[0]->kernel_index].kind != ImplKind::TileProgram) continue;
            const DType sdt = plan.tensors[ld.slot_tensor.tensor].dtype;
            if (sdt == DType::F16 || sdt == DType::BF16) continue;
            ds->load = &ld;
            cd.dev_select = ds;
            ld.dev_deferred = true;
        }
    }
    if (n.body) find_dev_selects(plan, impls, *n.body);
    for (auto& c : n.children) find_dev_selects(plan, impls, *c);
}

// Whether the walk depends on data that the replay key (logged symbols, axis sizes, ragged length sums, CSR
// contents) does not cover: slots (set from tensors or by the caller) read by a cond.
bool data_dependent(const Node& n) {
    switch (n.kind) {
        case Node::Kind::Cond:
            if (n.dev_select) return false;
            if (expr_mentions(n.pred.get(), Expr::Op::Slot, true, 0) ||
                expr_mentions(n.pred.get(), Expr::Op::TaskParam, true, 0))
                return true;
            return data_dependent(*n.then_n) || data_dependent(*n.else_n);
        case Node::Kind::SlotLoad:
            return !n.dev_deferred;
        case Node::Kind::SlotSet:
            return true;
        case Node::Kind::Select:
            return data_dependent(*n.body);
        case Node::Kind::ParallelFor:
        case Node::Kind::ForEach:
        case Node::Kind::Send:
        case Node::Kind::Consume:
            return data_dependent(*n.body);
        case Node::Kind::Combine:
        case Node::Kind::Sequential:
        case Node::Kind::Pipeline:
            for (auto& c : n.children)
                if (data_dependent(*c)) return true;
            return false;
        default:
            return false;
    }
}

}  // namespace

uint64_t reference_kernel_cycles(const KernelDef& kd) {
    KernelWalker w(kd, nullptr);
    w.run();
    return w.cycles;
}

std::unique_ptr<Program> compile_program(const char* text, size_t len, int device) {
    auto prog = std::make_unique<Program>();
    try {
        prog->plan = parse_plan(text, len);
    } catch (const Error&) {
        throw;
    } catch (const std::exception& e) {
        throw Error(PTOWSP_ERR_PLAN, e.what());
    }
    Plan& plan = prog->plan;
    prog->device = device;
    prog->impls.resize(plan.kernels.size());
    for (size_t i = 0; i < plan.kernels.size(); ++i) {
        const KernelDef& kd = plan.kernels[i];
        KernelImpl& ki = prog->impls[i];
        if (!kd.builtin.empty()) {
            setup_builtin(kd, ki);
            continue;
        }
        if (kd.has_cpp_body)
            throw Error(PTOWSP_ERR_UNSUPPORTED,
                        "kernel '" + kd.name + "' has a CPU C++ body (cpp_src/cpp_file_src); the cuda_sm100a target "
                        "runs only pto.* kernels and its built-ins");
        KernelWalker w(kd, &ki.tp);
        w.run();
        ki.cycles = w.cycles;
        ki.param_read = w.read;
        ki.param_write = w.written;
        ki.tp_smem = ki.tp.smem_words * 4;
        ki.tp_ok = w.error.empty() && ki.tp_smem <= dev::tile_program_max_smem();
        ki.tp_error = !w.error.empty() ? w.error
                      : (ki.tp_ok ? "" : "tiles need " + std::to_string(ki.tp_smem) + " B of shared memory");
        if (is_rmsnorm(kd)) ki.kind = ImplKind::RmsNorm;
        else if (is_softmax(kd)) ki.kind = ImplKind::Softmax;
        else if (int f = matmul_form(kd)) ki.kind = f == 1 ? ImplKind::Matmul : ImplKind::MatmulAcc;
        else ki.kind = ImplKind::TileProgram;
        // the attention pattern runs fused on tcgen05, its stages built as the fallback for views it does not take
        if (ki.kind == ImplKind::TileProgram && w.error.empty() && match_attention(ki, kd) && split_stages(ki, kd)) {
            bool built = true;
            for (size_t si = 0; built && si < ki.stages.size(); ++si) {
                Stage& st = ki.stages[si];
                if (st.mm) continue;
                std::string note;
                const std::string name = "ptowsp_st_k" + std::to_string(i) + "_" + std::to_string(si);
                if (build_stage_program(st.tp, kd, name, &st.cubin, &note)) st.jit_state = 2;
                else built = false;
            }
            if (built) {
                ki.kind = ImplKind::Attention;
                ki.jit_note = "fused attention on tcgen05 (the stages run views it does not take)";
                continue;
            }
            ki.stages.clear();
            ki.scratch_tiles.clear();
        }
        if (ki.kind == ImplKind::TileProgram && w.error.empty() && split_matmul_epilogue(ki, kd, static_cast<int>(i)))
            continue;
        // (only a complete tile program is cut: a walker error means an op is missing from it)
        if (ki.kind == ImplKind::TileProgram && w.error.empty() && split_stages(ki, kd)) {
            // stages (matmuls + fused row programs over HBM scratch) when the tiles exceed shared memory or a
            // contraction is large enough to want its own kernel; small kernels keep the one-launch tile program
            bool staged = !ki.tp_ok;
            for (const auto& st : ki.stages)
                if (st.mm && int64_t(st.m) * st.n * st.k >= int64_t(128) * 128 * 64) staged = true;
            for (size_t si = 0; staged && si < ki.stages.size(); ++si) {
                Stage& st = ki.stages[si];
                if (st.mm) continue;
                std::string note;
                const std::string name = "ptowsp_st_k" + std::to_string(i) + "_" + std::to_string(si);
                if (build_stage_program(st.tp, kd, name, &st.cubin, &note)) st.jit_state = 2;
                else staged = false;
            }
            if (staged) {
                ki.kind = ImplKind::Staged;
                ki.jit_note = "cut at its contractions: matmul kernels and fused row programs over HBM scratch";
                continue;
            }
            ki.stages.clear();
            ki.scratch_tiles.clear();
        }
        if (ki.kind == ImplKind::TileProgram && !ki.tp_ok)
            throw Error(PTOWSP_ERR_UNSUPPORTED, "kernel '" + kd.name + "': " + ki.tp_error);
        // a generic kernel gets its fused row kernel built now (NVRTC, no GPU needed), and so does a fast row op
        // whose tile width the hand-written kernel does not take; the others build theirs only if a launch falls
        // back to the tile program (unaligned views)
        const bool odd_width = (ki.kind == ImplKind::RmsNorm || ki.kind == ImplKind::Softmax) &&
                               !dev::row_width_supported(kd.params[0].v.cols);
        if (ki.kind == ImplKind::TileProgram || odd_width) jit_prepare(ki, kd, static_cast<int>(i));
    }
    prog->tensor_key_depth.assign(plan.tensors.size(), -1);
    collect_depths(plan, *plan.body, prog->tensor_key_depth);
    find_dev_selects(plan, prog->impls, *plan.body);
    prog->cacheable = !data_dependent(*plan.body);
    return prog;
}

std::string describe_program(const Program& p) {
    std::ostringstream o;
    o << "{\"name\":\"" << p.plan.name << "\",\"cacheable\":" << (p.cacheable ? "true" : "false")
      << ",\"window_tasks\":" << p.plan.schedule.window_tasks << ",\"dispatch\":\"" << p.plan.schedule.dispatch_policy
      << "\",\"num_targets\":" << p.plan.schedule.num_targets << ",\"kernels\":[";
    for (size_t i = 0; i < p.impls.size(); ++i) {
        if (i) o << ",";
        const KernelImpl& ki = p.impls[i];
        std::string note;
        for (char c : ki.jit_note.substr(0, 200)) note += (c == '"' || c == '\\' || c < 32) ? ' ' : c;
        const char* row = ki.jit_state == 1 ? "loaded" : ki.jit_state == 2 ? "compiled" : ki.jit_state == 0 ? "not built" : "interpreter";
        o << "{\"name\":\"" << p.plan.kernels[i].name << "\",\"impl\":\"" << impl_name(ki.kind)
          << "\",\"cycles\":" << ki.cycles << ",\"tile_program_smem\":" << ki.tp_smem << ",\"row_kernel\":\"" << row
          << "\",\"row_kernel_note\":\"" << note << "\"";
        if (ki.kind == ImplKind::Staged || ki.kind == ImplKind::Attention) {  // e.g. ["matmul 128x256x128 tcgen05", "rows 128", ...]
            o << ",\"stages\":[";
            for (size_t si = 0; si < ki.stages.size(); ++si) {
                const Stage& st = ki.stages[si];
                o << (si ? "," : "") << "\"";
                if (!st.mm) {
                    o << "rows " << st.rows;
                } else {
                    o << "matmul " << st.m << "x" << st.n << "x" << st.k << (st.tc ? " tcgen05" : " cuda_cores");
                    if (st.tc && st.tn != st.n) o << " (" << st.n / st.tn << " tiles of " << st.tn << ")";
                }
                o << "\"";
            }
            o << "],\"scratch_tiles\":" << ki.scratch_tiles.size();
        }
        o << "}";
    }
    o << "]";
    if (p.cached) {
        o << ",\"waves\":" << p.cached->waves.size() << ",\"tasks\":" << p.cached->tasks;
    }
    if (!p.csp_mode.empty()) {  // a CSP pipeline body: device processes, or waves and why
        std::string m;
        for (char c : p.csp_mode.substr(0, 200)) m += (c == '"' || c == '\\' || c < 32) ? ' ' : c;
        o << ",\"csp\":\"" << m << "\"";
    }
    o << "}";
    return o.str();
}

}  // namespace ptowsp
