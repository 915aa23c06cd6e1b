// Workload plan model: the reference codegen ir::Module (include/pto/wsp/ir/
// codegen.hpp:20-77, workload.hpp, schedule.hpp) as read from a
// "ptowsp-plan/1" JSON document.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "json.hpp"

namespace ptowsp {

enum class DType : uint8_t { F16, BF16, F32, F64, I8, I16, I32, I64, U8, U16, U32, U64, Bool };

DType parse_dtype(const std::string& s);
int dtype_bytes(DType d);
const char* dtype_name(DType d);

// Scalar expressions (include/pto/wsp/ir/scalar_expr.hpp:60-260).
struct Expr {
    enum class Op : uint8_t { Lit, Axis, Sym, Tag, Slot, TaskParam, Unary, Binary, Ternary, Cast };
    enum class Ty : uint8_t { Bool, I64, U64 };
    Op op = Op::Lit;
    Ty ty = Ty::I64;
    uint64_t v = 0;          // literal bits / axis id / symbol id / slot index / task param index
    std::string fn;          // unary / binary operator
    std::shared_ptr<Expr> a, b, c;
};
using ExprPtr = std::shared_ptr<Expr>;

struct IndexExpr {
    bool is_var = false;
    std::string var;
    int64_t c = 0;
};

struct TensorArg {  // CodegenTensorArg (codegen.hpp:34-40)
    std::string param;
    uint32_t tensor = 0;
    int base_rank = 0;
    int view_rank = 0;
    std::vector<IndexExpr> index;
};

struct ArgSpec {  // CodegenAxisArg (codegen.hpp:28-32)
    enum class Kind : uint8_t { Var, Sym, U64 } kind = Kind::U64;
    std::string var;
    uint64_t v = 0;
};

struct Axis {
    enum class Kind : uint8_t { Dense, DenseDyn, Ragged } kind = Kind::Dense;
    int64_t size = 0;
    uint64_t outer_sym = 0, lengths_sym = 0;
};

// CSP pipeline pieces (include/pto/wsp/ir/csp.hpp): channels by index within their pipeline.
struct ChannelDef {
    std::string name;
    int64_t capacity = 0;  // 0: rendezvous
};
struct ProcessDef {
    std::string name;
    std::vector<int> produces, consumes;  // channel indices
};

struct Node;

// A `P.when` tree over one slot that `slot_load_u64` fills from a tensor just before it, whose leaves are tasks of
// one kernel on the same views that differ only in their scalar args (the reference indexer's tiers): the walk
// places one task and the GPU picks the leaf's scalars from the tensor element itself (no host read of the data).
struct DevSelect {
    const Node* load = nullptr;             // the slot_load_u64 node
    std::vector<const Node*> leaves;        // task leaves in tree order
    // per cond of the tree (index order): comparison, which side the slot is on, the other operand, children
    // (>= 0: cond index, < 0: ~leaf index)
    std::vector<std::string> cmp;
    std::vector<uint8_t> slot_left;
    std::vector<const Expr*> other;
    std::vector<const Expr*> slot_expr;
    std::vector<int> then_c, else_c;
};

struct Node {
    enum class Kind : uint8_t { ParallelFor, ForEach, Task, Combine, Sequential, Cond, Select, SlotSet, SlotLoad,
                                Pipeline, Send, Consume };
    Kind kind = Kind::Task;
    // loops / select
    std::string var;
    Axis axis;
    std::shared_ptr<Node> body;
    uint64_t outer_sym = 0, indptr_sym = 0, indices_sym = 0;
    // combine / sequential
    std::vector<std::shared_ptr<Node>> children;
    // cond
    ExprPtr pred;
    std::shared_ptr<Node> then_n, else_n;
    // task
    std::string kernel;
    int kernel_index = -1;
    std::vector<ArgSpec> axis_args, scalar_args;
    std::vector<TensorArg> tensor_args;
    std::vector<int> param_to_arg;  // kernel tensor-param order -> index into tensor_args
    // slots
    uint32_t slot = 0;
    uint64_t slot_value = 0;
    TensorArg slot_tensor;
    int64_t row = 0, col = 0;
    // pipeline: `children` holds the process bodies, in process order
    std::vector<ChannelDef> channels;
    std::vector<ProcessDef> processes;
    // send (body = the task whose first axis arg is the token) / consume (var = the token's name, body)
    std::string channel_name;
    int channel = -1;
    // device-selected scalars: on the root cond of such a tree; the slot_load feeding it is deferred
    std::shared_ptr<DevSelect> dev_select;
    bool dev_deferred = false;
};
using NodePtr = std::shared_ptr<Node>;

struct ValueInfo {
    DType dtype = DType::F32;
    int rows = -1, cols = -1;  // -1: scalar
    bool is_tile() const { return rows >= 0; }
};

struct OpInfo {
    std::string kind;
    int result = -1;
    std::vector<int> operands;
    json::Value attrs;
};

struct KernelParam {
    std::string name;
    int id = 0;
    ValueInfo v;
    int tensor_index = -1;  // index among tensor params
    int scalar_index = -1;  // index among scalar params
};

struct KernelDef {
    std::string name;
    std::vector<KernelParam> params;
    std::map<int, ValueInfo> values;
    std::vector<OpInfo> ops;
    json::Value attrs;
    int num_tensor_params = 0, num_scalar_params = 0;
    std::string builtin;  // non-empty for the target's built-in custom kernels
    bool has_cpp_body = false;
    const KernelParam* param_by_id(int id) const {
        for (auto& p : params)
            if (p.id == id) return &p;
        return nullptr;
    }
};

struct TensorInfo {
    DType dtype = DType::F32;
    std::vector<int64_t> shape;
};

struct Schedule {
    std::string dispatch_policy;  // "" = none
    int num_targets = 0;
    ExprPtr dispatch_key;
    int64_t window_tasks = 0;  // 0 = unlimited
    bool window_supported = true;
    int streams = 0;
    std::vector<std::string> unsupported;
};

struct Plan {
    std::string name;
    std::vector<TensorInfo> tensors;
    std::vector<KernelDef> kernels;
    NodePtr body;
    Schedule schedule;
    int kernel_index(const std::string& n) const {
        for (size_t i = 0; i < kernels.size(); ++i)
            if (kernels[i].name == n) return static_cast<int>(i);
        return -1;
    }
};

Plan parse_plan(const char* text, size_t len);

uint64_t fnv1a_64(const std::string& s);

}  // namespace ptowsp
