// Plan parsing: JSON ("ptowsp-plan/1") -> ptowsp::Plan.  Also resolves task ->
// kernel bindings the way the reference emitter does (tensor args bound to
// kernel tensor params by name, pto_codegen.cpp:2550-2568).
#include "plan.hpp"

#include <algorithm>
#include <functional>
#include <stdexcept>

namespace ptowsp {

uint64_t fnv1a_64(const std::string& s) {
    uint64_t h = 0xCBF29CE484222325ULL;
    for (unsigned char c : s) {
        h ^= static_cast<uint64_t>(c);
        h *= 0x100000001B3ULL;
    }
    return h;
}

DType parse_dtype(const std::string& s) {
    if (s == "f16") return DType::F16;
    if (s == "bf16") return DType::BF16;
    if (s == "f32") return DType::F32;
    if (s == "f64") return DType::F64;
    if (s == "i8") return DType::I8;
    if (s == "i16") return DType::I16;
    if (s == "i32") return DType::I32;
    if (s == "i64") return DType::I64;
    if (s == "u8") return DType::U8;
    if (s == "u16") return DType::U16;
    if (s == "u32") return DType::U32;
    if (s == "u64") return DType::U64;
    if (s == "bool") return DType::Bool;
    throw std::runtime_error("plan: unsupported dtype " + s);
}

int dtype_bytes(DType d) {
    switch (d) {
        case DType::F16: case DType::BF16: case DType::I16: case DType::U16: return 2;
        case DType::F32: case DType::I32: case DType::U32: return 4;
        case DType::F64: case DType::I64: case DType::U64: return 8;
        case DType::I8: case DType::U8: case DType::Bool: return 1;
    }
    return 4;
}

const char* dtype_name(DType d) {
    switch (d) {
        case DType::F16: return "f16";
        case DType::BF16: return "bf16";
        case DType::F32: return "f32";
        case DType::F64: return "f64";
        case DType::I8: return "i8";
        case DType::I16: return "i16";
        case DType::I32: return "i32";
        case DType::I64: return "i64";
        case DType::U8: return "u8";
        case DType::U16: return "u16";
        case DType::U32: return "u32";
        case DType::U64: return "u64";
        case DType::Bool: return "bool";
    }
    return "?";
}

namespace {

Expr::Ty parse_ty(const std::string& s) {
    if (s == "bool") return Expr::Ty::Bool;
    if (s == "u64") return Expr::Ty::U64;
    return Expr::Ty::I64;
}

ExprPtr parse_expr(const json::Value& j) {
    auto e = std::make_shared<Expr>();
    const std::string& op = j.at("op").as_str();
    if (op == "lit") {
        e->op = Expr::Op::Lit;
        e->ty = parse_ty(j.at("type").as_str());
        e->v = j.at("v").as_u64();
    } else if (op == "axis") {
        e->op = Expr::Op::Axis;
        e->ty = Expr::Ty::I64;
        e->v = j.at("id").as_u64();
    } else if (op == "sym" || op == "tag") {
        e->op = op == "sym" ? Expr::Op::Sym : Expr::Op::Tag;
        e->ty = Expr::Ty::U64;
        e->v = j.at("id").as_u64();
    } else if (op == "slot") {
        e->op = Expr::Op::Slot;
        e->ty = parse_ty(j.at("type").as_str());
        e->v = j.at("i").as_u64();
    } else if (op == "task_param") {
        e->op = Expr::Op::TaskParam;
        e->ty = Expr::Ty::U64;
        e->v = j.at("i").as_u64();
    } else if (op == "un") {
        e->op = Expr::Op::Unary;
        e->fn = j.at("fn").as_str();
        e->a = parse_expr(j.at("a"));
    } else if (op == "bin") {
        e->op = Expr::Op::Binary;
        e->fn = j.at("fn").as_str();
        e->a = parse_expr(j.at("a"));
        e->b = parse_expr(j.at("b"));
    } else if (op == "tern") {
        e->op = Expr::Op::Ternary;
        e->c = parse_expr(j.at("c"));
        e->a = parse_expr(j.at("a"));
        e->b = parse_expr(j.at("b"));
    } else if (op == "cast") {
        e->op = Expr::Op::Cast;
        e->ty = parse_ty(j.at("type").as_str());
        e->a = parse_expr(j.at("a"));
    } else {
        throw std::runtime_error("plan: unknown scalar expr op " + op);
    }
    return e;
}

TensorArg parse_tensor_arg(const json::Value& j) {
    TensorArg t;
    t.param = j.at("param").as_str();
    t.tensor = static_cast<uint32_t>(j.at("tensor").as_i64());
    t.base_rank = static_cast<int>(j.at("base_rank").as_i64());
    t.view_rank = static_cast<int>(j.at("view_rank").as_i64());
    for (auto& ie : j.at("index").arr) {
        IndexExpr x;
        if (ie.has("var")) {
            x.is_var = true;
            x.var = ie.at("var").as_str();
        } else {
            x.c = ie.at("const").as_i64();
        }
        t.index.push_back(std::move(x));
    }
    return t;
}

ArgSpec parse_arg(const json::Value& j) {
    ArgSpec a;
    if (j.has("var")) {
        a.kind = ArgSpec::Kind::Var;
        a.var = j.at("var").as_str();
    } else if (j.has("sym")) {
        a.kind = ArgSpec::Kind::Sym;
        a.v = j.at("sym").as_u64();
    } else {
        a.kind = ArgSpec::Kind::U64;
        a.v = j.at("u64").as_u64();
    }
    return a;
}

NodePtr parse_node(const json::Value& j) {
    auto n = std::make_shared<Node>();
    const std::string& k = j.at("kind").as_str();
    if (k == "parallel_for" || k == "for_each") {
        n->kind = k == "parallel_for" ? Node::Kind::ParallelFor : Node::Kind::ForEach;
        n->var = j.at("var").as_str();
        const auto& ax = j.at("axis");
        const std::string& ak = ax.at("kind").as_str();
        if (ak == "dense") {
            n->axis.kind = Axis::Kind::Dense;
            n->axis.size = ax.at("size").as_i64();
        } else if (ak == "dense_dyn") {
            n->axis.kind = Axis::Kind::DenseDyn;
        } else if (ak == "ragged") {
            n->axis.kind = Axis::Kind::Ragged;
            n->axis.outer_sym = ax.at("outer_sym").as_u64();
            n->axis.lengths_sym = ax.at("lengths_sym").as_u64();
        } else {
            throw std::runtime_error("plan: Unsupported axis kind for parallel_for in codegen: " + ak);
        }
        n->body = parse_node(j.at("body"));
    } else if (k == "task") {
        n->kind = Node::Kind::Task;
        n->kernel = j.at("kernel").as_str();
        for (auto& a : j.at("axis_args").arr) n->axis_args.push_back(parse_arg(a));
        for (auto& a : j.at("scalar_args").arr) n->scalar_args.push_back(parse_arg(a));
        for (auto& a : j.at("tensor_args").arr) n->tensor_args.push_back(parse_tensor_arg(a));
    } else if (k == "combine" || k == "sequential") {
        n->kind = k == "combine" ? Node::Kind::Combine : Node::Kind::Sequential;
        for (auto& c : j.at("children").arr) n->children.push_back(parse_node(c));
    } else if (k == "cond") {
        n->kind = Node::Kind::Cond;
        n->pred = parse_expr(j.at("pred"));
        n->then_n = parse_node(j.at("then"));
        n->else_n = parse_node(j.at("else"));
    } else if (k == "select") {
        n->kind = Node::Kind::Select;
        n->var = j.at("var").as_str();
        n->outer_sym = j.at("outer_sym").as_u64();
        n->indptr_sym = j.at("indptr_sym").as_u64();
        n->indices_sym = j.at("indices_sym").as_u64();
        n->body = parse_node(j.at("body"));
    } else if (k == "slot_set") {
        n->kind = Node::Kind::SlotSet;
        n->slot = static_cast<uint32_t>(j.at("slot").as_i64());
        n->slot_value = j.at("value").as_u64();
    } else if (k == "slot_load") {
        n->kind = Node::Kind::SlotLoad;
        n->slot = static_cast<uint32_t>(j.at("slot").as_i64());
        n->slot_tensor = parse_tensor_arg(j.at("tensor_arg"));
        n->row = j.at("row").as_i64();
        n->col = j.at("col").as_i64();
    } else if (k == "pipeline") {
        n->kind = Node::Kind::Pipeline;
        std::map<std::string, int> index;
        for (auto& c : j.at("channels").arr) {
            ChannelDef cd;
            cd.name = c.at("name").as_str();
            cd.capacity = std::max<int64_t>(0, c.at("capacity").as_i64());
            index[cd.name] = static_cast<int>(n->channels.size());
            n->channels.push_back(std::move(cd));
        }
        auto resolve = [&](const std::string& name) {
            auto it = index.find(name);
            if (it == index.end()) throw std::runtime_error("CSPT codegen: unknown channel: " + name);
            return it->second;
        };
        for (auto& pj : j.at("processes").arr) {
            ProcessDef pd;
            pd.name = pj.at("name").as_str();
            for (auto& c : pj.at("produces").arr) pd.produces.push_back(resolve(c.as_str()));
            for (auto& c : pj.at("consumes").arr) pd.consumes.push_back(resolve(c.as_str()));
            n->processes.push_back(std::move(pd));
            n->children.push_back(parse_node(pj.at("body")));
        }
        // channels named by send / consume nodes of the process bodies
        std::function<void(Node&)> bind = [&](Node& x) {
            if (x.kind == Node::Kind::Send || x.kind == Node::Kind::Consume) x.channel = resolve(x.channel_name);
            if (x.kind == Node::Kind::Pipeline) throw std::runtime_error("CSPT codegen: nested pipeline");
            if (x.body) bind(*x.body);
            for (auto& c : x.children) bind(*c);
            if (x.then_n) bind(*x.then_n);
            if (x.else_n) bind(*x.else_n);
        };
        for (auto& c : n->children) bind(*c);
    } else if (k == "send") {
        n->kind = Node::Kind::Send;
        n->channel_name = j.at("channel").as_str();
        n->body = parse_node(j.at("value"));
        if (n->body->kind != Node::Kind::Task) throw std::runtime_error("CSPT codegen: send value must be a Task node");
    } else if (k == "consume") {
        n->kind = Node::Kind::Consume;
        n->channel_name = j.at("channel").as_str();
        n->var = j.at("var").as_str();
        n->body = parse_node(j.at("body"));
    } else {
        throw std::runtime_error("plan: Unhandled workload node kind " + k);
    }
    return n;
}

KernelDef parse_kernel(const json::Value& j) {
    KernelDef kd;
    kd.name = j.at("name").as_str();
    for (auto& v : j.at("values").arr) {
        ValueInfo vi;
        vi.dtype = parse_dtype(v.arr.at(1).as_str());
        vi.rows = static_cast<int>(v.arr.at(2).as_i64());
        vi.cols = static_cast<int>(v.arr.at(3).as_i64());
        kd.values[static_cast<int>(v.arr.at(0).as_i64())] = vi;
    }
    for (auto& p : j.at("params").arr) {
        KernelParam kp;
        kp.name = p.at("name").as_str();
        kp.id = static_cast<int>(p.at("id").as_i64());
        auto it = kd.values.find(kp.id);
        if (it == kd.values.end()) throw std::runtime_error("plan: Kernel param missing from values map");
        kp.v = it->second;
        if (kp.v.is_tile()) kp.tensor_index = kd.num_tensor_params++;
        else kp.scalar_index = kd.num_scalar_params++;
        kd.params.push_back(std::move(kp));
    }
    for (auto& o : j.at("ops").arr) {
        OpInfo oi;
        oi.kind = o.at("kind").as_str();
        oi.result = static_cast<int>(o.at("result").as_i64());
        for (auto& x : o.at("operands").arr) oi.operands.push_back(static_cast<int>(x.as_i64()));
        if (auto* a = o.get("attrs")) oi.attrs = *a;
        kd.ops.push_back(std::move(oi));
    }
    if (auto* a = j.get("attrs")) kd.attrs = *a;
    if (auto* b = kd.attrs.get("builtin")) kd.builtin = b->as_str();
    if (auto* src = kd.attrs.get("cpp_src")) {
        kd.has_cpp_body = true;
        // Built-in marker line: "// ptowsp-builtin: <name>"
        const std::string& s = src->as_str();
        size_t pos = s.find("// ptowsp-builtin:");
        if (pos != std::string::npos && kd.builtin.empty()) {
            size_t e = s.find('\n', pos);
            std::string nm = s.substr(pos + 18, e == std::string::npos ? std::string::npos : e - pos - 18);
            size_t a = nm.find_first_not_of(" \t"), b = nm.find_last_not_of(" \t\r");
            if (a != std::string::npos) kd.builtin = nm.substr(a, b - a + 1);
        }
    }
    if (kd.attrs.get("cpp_file_src")) kd.has_cpp_body = true;
    return kd;
}

void bind_tasks(Plan& plan, Node& n) {
    switch (n.kind) {
        case Node::Kind::ParallelFor:
        case Node::Kind::ForEach:
        case Node::Kind::Select:
        case Node::Kind::Send:
        case Node::Kind::Consume:
            bind_tasks(plan, *n.body);
            break;
        case Node::Kind::Combine:
        case Node::Kind::Sequential:
        case Node::Kind::Pipeline:
            for (auto& c : n.children) bind_tasks(plan, *c);
            break;
        case Node::Kind::Cond:
            bind_tasks(plan, *n.then_n);
            bind_tasks(plan, *n.else_n);
            break;
        case Node::Kind::Task: {
            n.kernel_index = plan.kernel_index(n.kernel);
            if (n.kernel_index < 0) throw std::runtime_error("plan: Missing kernel def for task: " + n.kernel);
            const KernelDef& kd = plan.kernels[n.kernel_index];
            n.param_to_arg.assign(kd.num_tensor_params, -1);
            for (const auto& p : kd.params) {
                if (p.tensor_index < 0) continue;
                int found = -1;
                for (size_t i = 0; i < n.tensor_args.size(); ++i)
                    if (n.tensor_args[i].param == p.name) found = static_cast<int>(i);
                if (found < 0) throw std::runtime_error("plan: Missing tensor arg for param: " + p.name);
                const auto& ta = n.tensor_args[found];
                if (ta.tensor >= plan.tensors.size()) throw std::runtime_error("plan: tensor id out of range");
                if (static_cast<int>(ta.index.size()) > static_cast<int>(plan.tensors[ta.tensor].shape.size()))
                    throw std::runtime_error("plan: view has more indices than its tensor has dims");
                n.param_to_arg[p.tensor_index] = found;
            }
            if (static_cast<int>(n.scalar_args.size()) != kd.num_scalar_params)
                throw std::runtime_error("plan: scalar arg count mismatch for task " + n.kernel);
            break;
        }
        case Node::Kind::SlotLoad:
            if (n.slot_tensor.tensor >= plan.tensors.size()) throw std::runtime_error("plan: tensor id out of range");
            break;
        default:
            break;
    }
}

}  // namespace

Plan parse_plan(const char* text, size_t len) {
    json::Value j = json::parse(text, len);
    if (!j.is_obj() || !j.has("format") || j.at("format").as_str() != "ptowsp-plan/1")
        throw std::runtime_error("plan: not a ptowsp-plan/1 document");
    Plan p;
    p.name = j.at("name").as_str();
    for (auto& t : j.at("tensors").arr) {
        TensorInfo ti;
        ti.dtype = parse_dtype(t.at("dtype").as_str());
        for (auto& d : t.at("shape").arr) ti.shape.push_back(d.as_i64());
        p.tensors.push_back(std::move(ti));
    }
    for (auto& k : j.at("kernels").arr) p.kernels.push_back(parse_kernel(k));
    p.body = parse_node(j.at("body"));
    if (auto* s = j.get("schedule")) {
        if (auto* d = s->get("dispatch"); d && d->is_obj()) {
            p.schedule.dispatch_policy = d->at("policy").as_str();
            p.schedule.num_targets = static_cast<int>(d->at("num_targets").as_i64());
            if (auto* k = d->get("key"); k && k->is_obj()) p.schedule.dispatch_key = parse_expr(*k);
            bool key_required = p.schedule.dispatch_policy == "affinity" || p.schedule.dispatch_policy == "hash" ||
                                p.schedule.dispatch_policy == "custom";
            if (key_required && !p.schedule.dispatch_key)
                throw std::runtime_error(
                    "dispatch policy requires ScalarExpr key (string-eval is not supported in v9 codegen-first)");
        }
        if (auto* w = s->get("task_window"); w && w->is_obj()) {
            bool ok = w->at("unit").as_str() == "tasks" && w->at("overflow").as_str() == "stall";
            if (ok) p.schedule.window_tasks = std::max<int64_t>(w->at("size").as_i64(), 0);
            else p.schedule.unsupported.push_back("task_window(non-stall or non-tasks)");
        }
        if (auto* st = s->get("streams")) p.schedule.streams = static_cast<int>(st->as_i64());
        if (auto* u = s->get("unsupported"); u && u->is_arr())
            for (auto& x : u->arr) p.schedule.unsupported.push_back(x.as_str());
    }
    bind_tasks(p, *p.body);
    return p;
}

}  // namespace ptowsp
