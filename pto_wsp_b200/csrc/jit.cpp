// Row-program compiler: generic tile programs lowered to fused CUDA kernels.
//
// A tile program (the emitter's op set, src/python/pto_codegen.cpp:785-1231) is
// "row-local" when every instruction works on whole rows of its tiles: loads
// and stores of full tiles, element-wise binary / scalar / exp / rsqrt ops,
// row-broadcast operands ([R,1] tiles) and row reductions.  Such a program --
// RMSNorm or softmax of any width, scale/shift chains, row normalisations --
// is lowered to one straight-line kernel specialised on its shapes, op
// sequence and parameter types: one warp per tile row, the row's elements in
// registers (lane l holds columns l, l+32, ...), reductions by warp shuffles,
// no shared memory and no block barriers.  The source is compiled at the first
// launch with NVRTC (loaded with dlopen) for sm_100a and loaded through the
// driver API; a program that is not row-local, or any failure on the way,
// keeps the shared-memory tile-program interpreter (rows.cu), which is also a
// GPU kernel.  Element-wise results match the interpreter bit for bit; row
// reductions add in tree order instead of column order (the hand-written row
// kernels do the same), within the fp32 tolerance.
#include "jit.hpp"

#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <sstream>
#include <string>
#include <unordered_map>
#include <vector>

namespace ptowsp::jit {

namespace {

using namespace dev;

constexpr int kMaxCols = 1024;     // a lane holds at most 32 elements of one tile row
constexpr int kMaxRegWords = 160;  // per lane, over all full-width tiles of the program (255 registers at most)

// ---- NVRTC, resolved at run time (no link-time dependency) ----
using nvrtcProgram_t = void*;
struct Nvrtc {
    int (*create)(nvrtcProgram_t*, const char*, const char*, int, const char* const*, const char* const*) = nullptr;
    int (*compile)(nvrtcProgram_t, int, const char* const*) = nullptr;
    int (*log_size)(nvrtcProgram_t, size_t*) = nullptr;
    int (*log)(nvrtcProgram_t, char*) = nullptr;
    int (*cubin_size)(nvrtcProgram_t, size_t*) = nullptr;
    int (*cubin)(nvrtcProgram_t, char*) = nullptr;
    int (*destroy)(nvrtcProgram_t*) = nullptr;
    bool ok = false;
};

const Nvrtc& nvrtc() {
    static Nvrtc n;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* names[] = {"libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so.12",
                               "/usr/local/cuda/lib64/libnvrtc.so"};
        void* h = nullptr;
        for (const char* nm : names)
            if ((h = dlopen(nm, RTLD_NOW | RTLD_LOCAL)) != nullptr) break;
        if (!h) return;
        auto sym = [&](const char* s) { return dlsym(h, s); };
        n.create = reinterpret_cast<decltype(n.create)>(sym("nvrtcCreateProgram"));
        n.compile = reinterpret_cast<decltype(n.compile)>(sym("nvrtcCompileProgram"));
        n.log_size = reinterpret_cast<decltype(n.log_size)>(sym("nvrtcGetProgramLogSize"));
        n.log = reinterpret_cast<decltype(n.log)>(sym("nvrtcGetProgramLog"));
        n.cubin_size = reinterpret_cast<decltype(n.cubin_size)>(sym("nvrtcGetCUBINSize"));
        n.cubin = reinterpret_cast<decltype(n.cubin)>(sym("nvrtcGetCUBIN"));
        n.destroy = reinterpret_cast<decltype(n.destroy)>(sym("nvrtcDestroyProgram"));
        n.ok = n.create && n.compile && n.log_size && n.log && n.cubin_size && n.cubin && n.destroy;
    });
    return n;
}

// ---- driver API entry points ----
struct Driver {
    CUresult (*load)(CUmodule*, const void*) = nullptr;
    CUresult (*get)(CUfunction*, CUmodule, const char*) = nullptr;
    CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream,
                       void**, void**) = nullptr;
    bool ok = false;
};

const Driver& driver() {
    static Driver d;
    static std::once_flag once;
    std::call_once(once, [] {
        auto entry = [](const char* name) -> void* {
            void* p = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
                return nullptr;
            return p;
        };
        d.load = reinterpret_cast<decltype(d.load)>(entry("cuModuleLoadData"));
        d.get = reinterpret_cast<decltype(d.get)>(entry("cuModuleGetFunction"));
        d.launch = reinterpret_cast<decltype(d.launch)>(entry("cuLaunchKernel"));
        d.ok = d.load && d.get && d.launch;
    });
    return d;
}

const char* kPrelude = R"(
typedef long long int64_t;
typedef unsigned long long uint64_t;
typedef int int32_t;
typedef unsigned int uint32_t;
struct ParamDesc { char* base; int64_t s3, s4; int64_t numel_span; int rows, cols; int type; int elem_bytes; };
struct TaskBatch { const int64_t* rec; int64_t ntasks; int stride; int nparams, naxis, nscalar; ParamDesc p[MAXP]; int* err; };
__device__ __forceinline__ float h2f(unsigned short h) { float f; asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h)); return f; }
__device__ __forceinline__ unsigned short f2h(float f) { unsigned short h; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f)); return h; }
)";

// Load expression of element `off` of param p (type `pt`) as the 32-bit word `word` (load_elem_w semantics).
std::string load_expr(int pt, int word, const std::string& p, const std::string& off) {
    const std::string fe = [&] {
        switch (pt) {
            case PT_F32: return "((const float*)" + p + ".base)[" + off + "]";
            case PT_F16: return "h2f(((const unsigned short*)" + p + ".base)[" + off + "])";
            case PT_I32: return "(float)((const int*)" + p + ".base)[" + off + "]";
            case PT_U32: return "(float)((const unsigned*)" + p + ".base)[" + off + "]";
            case PT_I64: return "(float)((const long long*)" + p + ".base)[" + off + "]";
            case PT_U64: return "(float)((const unsigned long long*)" + p + ".base)[" + off + "]";
            default: return std::string("0.f");
        }
    }();
    if (word == W_F32) return "__float_as_uint(" + fe + ")";
    switch (pt) {
        case PT_I32: case PT_U32: return "((const unsigned*)" + p + ".base)[" + off + "]";
        case PT_I64: case PT_U64: return "(unsigned)((const unsigned long long*)" + p + ".base)[" + off + "]";
        case PT_F32: return "(unsigned)(int)((const float*)" + p + ".base)[" + off + "]";
        case PT_F16: return "(unsigned)(int)h2f(((const unsigned short*)" + p + ".base)[" + off + "])";
        default: return "0u";
    }
}

// Store statement of word `w` (type `word`) to element `off` of param p (store_elem semantics).
std::string store_stmt(int pt, int word, const std::string& p, const std::string& off, const std::string& w) {
    const std::string f = word == W_F32 ? "__uint_as_float(" + w + ")"
                                        : (word == W_I32 ? "(float)(int)(" + w + ")" : "(float)(" + w + ")");
    switch (pt) {
        case PT_F32: return "((float*)" + p + ".base)[" + off + "] = " + f + ";";
        case PT_F16: return "((unsigned short*)" + p + ".base)[" + off + "] = f2h(" + f + ");";
        case PT_I32: return "((int*)" + p + ".base)[" + off + "] = " + (word == W_F32 ? "(int)" + f : "(int)(" + w + ")") + ";";
        case PT_U32: return "((unsigned*)" + p + ".base)[" + off + "] = " + (word == W_F32 ? "(unsigned)" + f : "(" + w + ")") + ";";
        case PT_I64: return "((long long*)" + p + ".base)[" + off + "] = " +
                            (word == W_F32 ? "(long long)" + f : "(long long)(int)(" + w + ")") + ";";
        case PT_U64: return "((unsigned long long*)" + p + ".base)[" + off + "] = " +
                            (word == W_F32 ? "(unsigned long long)" + f : "(unsigned long long)(" + w + ")") + ";";
        default: return ";";
    }
}

std::string bin_expr(int word, int sub, const std::string& a, const std::string& b) {
    if (word == W_F32) {
        const std::string fa = "__uint_as_float(" + a + ")", fb = "__uint_as_float(" + b + ")";
        switch (sub) {
            case BIN_ADD: return "__float_as_uint(__fadd_rn(" + fa + ", " + fb + "))";
            case BIN_SUB: return "__float_as_uint(__fsub_rn(" + fa + ", " + fb + "))";
            case BIN_MUL: return "__float_as_uint(__fmul_rn(" + fa + ", " + fb + "))";
            case BIN_DIV: return "__float_as_uint(__fdiv_rn(" + fa + ", " + fb + "))";
            case BIN_MAX: return "__float_as_uint(fmaxf(" + fa + ", " + fb + "))";
            default: return "__float_as_uint(fminf(" + fa + ", " + fb + "))";
        }
    }
    const std::string ia = "(int)(" + a + ")", ib = "(int)(" + b + ")";
    switch (sub) {
        case BIN_ADD: return "(unsigned)(" + ia + " + " + ib + ")";
        case BIN_SUB: return "(unsigned)(" + ia + " - " + ib + ")";
        case BIN_MUL: return "(unsigned)(" + ia + " * " + ib + ")";
        case BIN_DIV: return "(unsigned)(" + ib + " ? " + ia + " / " + ib + " : 0)";
        case BIN_MAX: return "(unsigned)(" + ia + " > " + ib + " ? " + ia + " : " + ib + ")";
        default: return "(unsigned)(" + ia + " < " + ib + " ? " + ia + " : " + ib + ")";
    }
}

}  // namespace

int program_rows(const TileProgram& tp) {
    int R = 0;
    for (int i = 0; i < tp.nslots; ++i) R = std::max(R, tp.slots[i].rows);
    return R;
}

// A one-row tile in a program over R > 1 rows: the same for every row ([1,C] operands of column broadcasts).
static bool row_invariant(const TileProgram& tp, int slot) { return tp.slots[slot].rows == 1 && program_rows(tp) > 1; }

// Element offset of tile row r of a view: none for a row-invariant tile (row 0 of its view); element r of row 0 for
// a load marked transposed (in.k == 1, see normalize).
static std::string row_offset(const TileProgram& tp, int slot, const std::string& p, bool transposed = false) {
    if (transposed) return " + (int64_t)r * " + p + ".s4";
    return row_invariant(tp, slot) ? std::string() : " + (int64_t)r * " + p + ".s3";
}

// The emitter broadcasts a one-row [1, R] operand over rows too (TROWEXPAND*: when its length equals the row
// count, element r goes to row r).  Such a tile, loaded from a param and used only that way, becomes an [R, 1]
// tile whose load (marked in.k = 1) reads element r of the view's first row for row r.
static TileProgram normalize(const TileProgram& tp) {
    TileProgram out = tp;
    const int R = program_rows(tp);
    if (R <= 1) return out;
    for (int s = 0; s < tp.nslots; ++s) {
        if (tp.slots[s].rows != 1 || tp.slots[s].cols != R) continue;
        int loads = 0, row_uses = 0, other = 0, ld = -1;
        for (int i = 0; i < tp.ninstr; ++i) {
            const TPInstr& in = tp.ins[i];
            // the slot fields each op uses (the others are left at zero)
            const bool d = in.op != TP_STORE && in.dst == s;
            const bool a = in.op != TP_LOAD && in.a == s;
            const bool b = (in.op == TP_BIN || in.op == TP_MATMUL) && in.b == s;
            if (in.op == TP_LOAD && d) {
                ++loads;
                ld = i;
            } else if (in.op == TP_BIN && in.mode == MODE_ROW && b && !a && !d) {
                ++row_uses;
            } else if (d || a || b) {
                ++other;
            }
        }
        if (loads != 1 || row_uses == 0 || other) continue;
        out.slots[s].rows = R;
        out.slots[s].cols = 1;
        out.ins[ld].rows = R;
        out.ins[ld].cols = 1;
        out.ins[ld].k = 1;
    }
    return out;
}

bool row_local(const TileProgram& tp_in, std::string* why) {
    const TileProgram tp = normalize(tp_in);
    auto fail = [&](const std::string& m) {
        if (why) *why = m;
        return false;
    };
    if (tp.ninstr <= 0 || tp.nslots <= 0) return fail("empty program");
    const int R = program_rows(tp);
    int words = 0;
    for (int i = 0; i < tp.nslots; ++i) {
        const TPSlot& s = tp.slots[i];
        if (s.rows != R && s.rows != 1) return fail("tiles of different row counts");
        if (s.cols < 1 || s.cols > kMaxCols) return fail("tile wider than 1024 columns");
        if (s.cols > 1) words += (s.cols + 31) / 32;
    }
    if (R < 1) return fail("no rows");
    if (words > kMaxRegWords) return fail("too many tile elements per lane");
    auto inv = [&](int slot) { return row_invariant(tp, slot); };
    for (int ii = 0; ii < tp.ninstr; ++ii) {
        const TPInstr& in = tp.ins[ii];
        switch (in.op) {
            case TP_LOAD: {
                const TPSlot& d = tp.slots[in.dst];
                if (in.rows != d.rows || in.cols != d.cols) return fail("partial-tile load");
                break;
            }
            case TP_STORE: {
                const TPSlot& a = tp.slots[in.a];
                if (in.rows != a.rows || in.cols != a.cols) return fail("partial-tile store");
                if (inv(in.a)) return fail("store of a one-row tile from a many-row program");
                break;
            }
            case TP_MOV: case TP_BINS: case TP_EXP: case TP_RSQRT: {
                const TPSlot &d = tp.slots[in.dst], &a = tp.slots[in.a];
                if (d.cols != a.cols || inv(in.dst) != inv(in.a)) return fail("shape change in an element-wise op");
                break;
            }
            case TP_BIN: {
                const TPSlot &d = tp.slots[in.dst], &a = tp.slots[in.a], &b = tp.slots[in.b];
                if (d.cols != a.cols || inv(in.dst) != inv(in.a)) return fail("shape change in a binary op");
                if (in.mode == MODE_FULL && (b.cols != d.cols || inv(in.b) != inv(in.dst)))
                    return fail("binary op on different shapes");
                if (in.mode == MODE_ROW && (b.cols != 1 || inv(in.b) != inv(in.dst))) return fail("row broadcast of a wide tile");
                if (in.mode == MODE_COL && (!inv(in.b) || b.cols != d.cols || inv(in.dst)))
                    return fail("column broadcast of a many-row tile");
                break;
            }
            case TP_ROWSUM: case TP_ROWMAX: case TP_ROWMEAN: {
                if (tp.slots[in.dst].cols != 1) return fail("row reduction into a wide tile");
                if (tp.slots[in.a].word != W_F32) return fail("integer row reduction");
                if (inv(in.dst) != inv(in.a)) return fail("row reduction across tile shapes");
                break;
            }
            default: return fail("op outside the row-local set");
        }
    }
    return true;
}

namespace {

// The scalar kernel of the row program: one warp per tile row, lane l holds columns l, l+32, ... (4-byte accesses,
// any strides).
void emit_row_kernel(std::ostringstream& o, const TileProgram& tp, const int* param_types, const std::string& name) {
    const int R = program_rows(tp);
    auto nwords = [&](int cols) { return (cols + 31) / 32; };
    o << "extern \"C\" __global__ void __launch_bounds__(256) " << name << "(TaskBatch b) {\n";
    o << "  const int lane = threadIdx.x & 31;\n";
    o << "  const int64_t nrows = b.ntasks * " << R << "LL;\n";
    o << "  for (int64_t g = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5); g < nrows; g += (int64_t)gridDim.x * 8) {\n";
    o << "    const int64_t task = g / " << R << "; const int r = (int)(g - task * " << R << ");\n";
    o << "    const int64_t* rec = b.rec + task * b.stride;\n";
    for (int i = 0; i < tp.nslots; ++i) {
        const TPSlot& sl = tp.slots[i];
        if (sl.cols > 1) o << "    unsigned s" << i << "[" << nwords(sl.cols) << "];\n";
        else o << "    unsigned s" << i << " = 0u;\n";
    }
    auto elem = [&](int slot, const std::string& j) {
        return tp.slots[slot].cols > 1 ? "s" + std::to_string(slot) + "[" + j + "]" : "s" + std::to_string(slot);
    };
    const std::string col = "(lane + 32 * j)";  // column of register word j of a lane
    for (int ii = 0; ii < tp.ninstr; ++ii) {
        const TPInstr& in = tp.ins[ii];
        o << "    { // instruction " << ii << "\n";
        switch (in.op) {
            case TP_LOAD:
            case TP_STORE: {
                const bool load = in.op == TP_LOAD;
                const int slot = load ? in.dst : in.a;
                const TPSlot& t = tp.slots[slot];
                const int pt = param_types[in.param];
                const std::string p = "b.p[" + std::to_string(in.param) + "]";
                o << "      const int64_t base = rec[" << in.param << "]" << row_offset(tp, slot, p, load && in.k == 1) << ";\n";
                const int nj = (t.cols + 31) / 32;
                o << "      #pragma unroll\n      for (int j = 0; j < " << nj << "; ++j) {\n";
                o << "        const int c = lane + 32 * j;" << (load ? " unsigned w = 0u;" : "") << "\n";
                o << "        if (c < " << t.cols << ") { const int64_t off = base + (int64_t)c * " << p << ".s4;\n";
                if (load) {
                    o << "          if (off >= 0 && off < " << p << ".numel_span) w = " << load_expr(pt, t.word, p, "off") << ";\n";
                } else {
                    o << "          if (off >= 0 && off < " << p << ".numel_span) { "
                      << store_stmt(pt, t.word, p, "off", t.cols > 1 ? elem(slot, "j") : elem(slot, "0")) << " }\n";
                }
                o << "          else atomicOr(b.err, " << kErrBounds << "); }\n";
                if (load) {
                    if (t.cols > 1) o << "        " << elem(slot, "j") << " = w;\n";
                    else o << "        if (j == 0) " << elem(slot, "0") << " = __shfl_sync(0xffffffffu, w, 0);\n";
                }
                o << "      }\n";
                break;
            }
            case TP_MOV: case TP_BIN: case TP_BINS: case TP_EXP: case TP_RSQRT: {
                const TPSlot& d = tp.slots[in.dst];
                const int nj = d.cols > 1 ? nwords(d.cols) : 1;
                if (in.op == TP_BINS) {
                    // the scalar operand as the op's word type (TP_BINS semantics of the interpreter)
                    const bool fw = d.word == W_F32;
                    if (in.scalar_src >= 0) {
                        o << "      const unsigned long long raw = (unsigned long long)rec[b.nparams + b.naxis + " << in.scalar_src
                          << "];\n";
                        const int st = tp.scalar_types[in.scalar_src];
                        if (st == 0) o << (fw ? "      const unsigned ws = (unsigned)raw;\n"
                                              : "      const unsigned ws = (unsigned)(int)__uint_as_float((unsigned)raw);\n");
                        else if (st == 2) o << (fw ? "      const unsigned ws = __float_as_uint((float)(long long)raw);\n"
                                                   : "      const unsigned ws = (unsigned)(int)raw;\n");
                        else o << (fw ? "      const unsigned ws = __float_as_uint((float)(int)raw);\n"
                                      : "      const unsigned ws = (unsigned)(int)raw;\n");
                    } else {
                        unsigned fbits;
                        std::memcpy(&fbits, &in.fval, 4);
                        o << "      const unsigned ws = "
                          << (fw ? std::to_string(fbits) + "u" : "(unsigned)(" + std::to_string(in.ival) + ")") << ";\n";
                    }
                }
                o << "      #pragma unroll\n      for (int j = 0; j < " << nj << "; ++j) {\n";
                std::string rhs;
                const std::string a = elem(in.a, "j");
                if (in.op == TP_MOV) rhs = a;
                else if (in.op == TP_BIN) rhs = bin_expr(d.word, in.sub, a, in.mode == MODE_ROW ? elem(in.b, "0") : elem(in.b, "j"));
                else if (in.op == TP_BINS) rhs = in.scalar_first ? bin_expr(d.word, in.sub, "ws", a) : bin_expr(d.word, in.sub, a, "ws");
                else if (in.op == TP_EXP) rhs = "__float_as_uint(expf(__uint_as_float(" + a + ")))";
                else rhs = "__float_as_uint(__fdiv_rn(1.0f, sqrtf(__uint_as_float(" + a + "))))";
                o << "        " << elem(in.dst, "j") << " = " << rhs << ";\n";
                o << "      }\n";
                break;
            }
            case TP_ROWSUM: case TP_ROWMAX: case TP_ROWMEAN: {
                const TPSlot& a = tp.slots[in.a];
                const int nj = a.cols > 1 ? nwords(a.cols) : 1;
                const bool mx = in.op == TP_ROWMAX;
                o << "      float acc = " << (mx ? "-__int_as_float(0x7f800000)" : "0.f") << ";\n";
                o << "      #pragma unroll\n      for (int j = 0; j < " << nj << "; ++j)\n";
                o << "        if (" << (a.cols > 1 ? col : std::string("lane")) << " < " << (a.cols > 1 ? a.cols : 1) << ") acc = "
                  << (mx ? "fmaxf(acc, __uint_as_float(" + elem(in.a, "j") + "))"
                         : "__fadd_rn(acc, __uint_as_float(" + elem(in.a, "j") + "))")
                  << ";\n";
                o << "      #pragma unroll\n      for (int o = 16; o > 0; o >>= 1) acc = "
                  << (mx ? "fmaxf(acc, __shfl_xor_sync(0xffffffffu, acc, o))" : "__fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o))")
                  << ";\n";
                if (in.op == TP_ROWMEAN) o << "      acc = __fdiv_rn(acc, (float)" << in.k << ");\n";
                o << "      " << elem(in.dst, "0") << " = __float_as_uint(acc);\n";
                break;
            }
            default: break;
        }
        o << "    }\n";
    }
    o << "  }\n}\n";
}

// Lanes per row for the vector kernel: the power of two L that leaves the fewest lanes idle on `quads`
// 16-byte column groups, with at most 8 quads per lane (32 registers per tile); ties go to the larger L.
int lanes_per_row(int quads) {
    int best = 32, waste = 1 << 30;
    for (int L = 32; L >= 1; L >>= 1) {
        const int per = (quads + L - 1) / L;
        if (per > 8) break;
        const int w = per * L - quads;
        if (w < waste) {
            waste = w;
            best = L;
        }
    }
    return best;
}

// The vector kernel: each tile row is handled by a group of L lanes (32 / L rows per warp), lane `sub` of a
// group holds the 4-column quads sub, sub + L, ... of the row; 16-byte (f32/i32) or 8-byte (f16) accesses;
// row reductions by shuffles inside the group.  Needs unit column strides and 16-byte-aligned rows.
void emit_group_kernel(std::ostringstream& o, const TileProgram& tp, const int* param_types, const std::string& name) {
    const int R = program_rows(tp);
    int cmax = 4;
    for (int i = 0; i < tp.nslots; ++i) cmax = std::max(cmax, tp.slots[i].cols);
    const int L = lanes_per_row((cmax + 3) / 4);
    const int RW = 32 / L;
    auto nq = [&](int cols) { return (cols + 4 * L - 1) / (4 * L); };  // quads per lane
    // occupancy: at most 256 / (words per lane + 36) blocks' worth of registers per thread, up to 4 blocks per SM
    // (the loop is latency-bound on its loads; 4 x 8 warps hides them, measured on softmax rows of 200 columns)
    const int minb = std::min(4, std::max(1, 256 / (4 * nq(cmax) + 36)));
    o << "extern \"C\" __global__ void __launch_bounds__(256, " << minb << ") " << name << "(TaskBatch b) {\n";
    bool bcast_load = false;
    for (int ii = 0; ii < tp.ninstr; ++ii)
        if (tp.ins[ii].op == TP_LOAD && tp.slots[tp.ins[ii].dst].cols == 1) bcast_load = true;
    o << "  const int lane = threadIdx.x & 31, sub = lane & " << L - 1 << ";\n";
    if (bcast_load) o << "  const int leader = lane & ~" << L - 1 << ";\n";
    o << "  const int64_t nrows = b.ntasks * " << R << "LL;\n";
    o << "  for (int64_t g0 = ((int64_t)blockIdx.x * 8 + (threadIdx.x >> 5)) * " << RW << "; g0 < nrows; g0 += (int64_t)gridDim.x * "
      << 8 * RW << ") {\n";
    o << "    const int64_t g = g0 + (lane >> " << __builtin_ctz(L) << "); const bool v = g < nrows;\n";
    o << "    const int64_t task = v ? g / " << R << " : 0; const int r = (int)(v ? g - task * " << R << " : 0);\n";
    o << "    const int64_t* rec = b.rec + task * b.stride;\n";
    for (int i = 0; i < tp.nslots; ++i) {
        const TPSlot& sl = tp.slots[i];
        if (sl.cols > 1) o << "    unsigned s" << i << "[" << 4 * nq(sl.cols) << "];\n";
        else o << "    unsigned s" << i << " = 0u;\n";
    }
    auto elem = [&](int slot, const std::string& j) {
        return tp.slots[slot].cols > 1 ? "s" + std::to_string(slot) + "[" + j + "]" : "s" + std::to_string(slot);
    };
    for (int ii = 0; ii < tp.ninstr; ++ii) {
        const TPInstr& in = tp.ins[ii];
        o << "    { // instruction " << ii << "\n";
        switch (in.op) {
            case TP_LOAD:
            case TP_STORE: {
                const bool load = in.op == TP_LOAD;
                const int slot = load ? in.dst : in.a;
                const TPSlot& t = tp.slots[slot];
                const int pt = param_types[in.param];
                const std::string p = "b.p[" + std::to_string(in.param) + "]";
                o << "      const int64_t base = rec[" << in.param << "]" << row_offset(tp, slot, p, load && in.k == 1) << ";\n";
                if (t.cols == 1) {  // [R,1]: the group leader's element, broadcast inside the group
                    if (load) {
                        o << "      unsigned w = 0u;\n";
                        o << "      if (v && sub == 0) { if (base >= 0 && base < " << p << ".numel_span) w = "
                          << load_expr(pt, t.word, p, "base") << "; else atomicOr(b.err, " << kErrBounds << "); }\n";
                        o << "      s" << slot << " = __shfl_sync(0xffffffffu, w, leader);\n";
                    } else {
                        o << "      if (v && sub == 0) { if (base >= 0 && base < " << p << ".numel_span) { "
                          << store_stmt(pt, t.word, p, "base", "s" + std::to_string(slot)) << " } else atomicOr(b.err, "
                          << kErrBounds << "); }\n";
                    }
                    break;
                }
                const bool half = pt == PT_F16;
                // the row is contiguous: one bounds check per row; quads below `full` are valid in every lane
                o << "      const bool rok = v && base >= 0 && base + " << t.cols << " <= " << p << ".numel_span;\n";
                o << "      if (v && !rok) atomicOr(b.err, " << kErrBounds << ");\n";
                o << "      #pragma unroll\n      for (int q = 0; q < " << nq(t.cols) << "; ++q) {\n";
                o << "        const int c0 = 4 * (sub + " << L << " * q);\n";
                o << "        if (rok && (q < " << t.cols / (4 * L) << " || c0 < " << t.cols << ")) { const int64_t off = base + c0;\n";
                o << "          {\n";
                if (load) {
                    if (half) {
                        o << "            const uint2 raw = __ldcs((const uint2*)(((const unsigned short*)" << p << ".base) + off));\n";
                        o << "            const unsigned short h[4] = {(unsigned short)(raw.x & 0xffffu), (unsigned short)(raw.x >> 16), "
                             "(unsigned short)(raw.y & 0xffffu), (unsigned short)(raw.y >> 16)};\n";
                        for (int e = 0; e < 4; ++e)
                            o << "            s" << slot << "[4 * q + " << e << "] = "
                              << (t.word == W_F32 ? "__float_as_uint(h2f(h[" + std::to_string(e) + "]))"
                                                  : "(unsigned)(int)h2f(h[" + std::to_string(e) + "])")
                              << ";\n";
                    } else {
                        o << "            const uint4 raw = __ldcs((const uint4*)(((const unsigned*)" << p << ".base) + off));\n";
                        const char* comp[4] = {"raw.x", "raw.y", "raw.z", "raw.w"};
                        for (int e = 0; e < 4; ++e) {
                            std::string w;
                            if (t.word == W_F32) {
                                if (pt == PT_F32) w = comp[e];
                                else if (pt == PT_I32) w = std::string("__float_as_uint((float)(int)") + comp[e] + ")";
                                else w = std::string("__float_as_uint((float)") + comp[e] + ")";
                            } else {
                                w = pt == PT_F32 ? std::string("(unsigned)(int)__uint_as_float(") + comp[e] + ")" : comp[e];
                            }
                            o << "            s" << slot << "[4 * q + " << e << "] = " << w << ";\n";
                        }
                    }
                } else {
                    std::string f[4];
                    for (int e = 0; e < 4; ++e) {
                        const std::string w = "s" + std::to_string(slot) + "[4 * q + " + std::to_string(e) + "]";
                        f[e] = t.word == W_F32 ? "__uint_as_float(" + w + ")"
                                               : (t.word == W_I32 ? "(float)(int)(" + w + ")" : "(float)(" + w + ")");
                        if (pt == PT_F16) f[e] = "f2h(" + f[e] + ")";
                        else if (pt == PT_F32) f[e] = "__float_as_uint(" + f[e] + ")";
                        else if (pt == PT_I32) f[e] = t.word == W_F32 ? "(unsigned)(int)" + f[e] : "(" + w + ")";
                        else f[e] = t.word == W_F32 ? "(unsigned)" + f[e] : "(" + w + ")";
                    }
                    if (half)
                        o << "            __stcs((uint2*)(((unsigned short*)" << p << ".base) + off), make_uint2((unsigned)" << f[0]
                          << " | ((unsigned)" << f[1] << " << 16), (unsigned)" << f[2] << " | ((unsigned)" << f[3] << " << 16)));\n";
                    else
                        o << "            __stcs((uint4*)(((unsigned*)" << p << ".base) + off), make_uint4(" << f[0] << ", " << f[1] << ", "
                          << f[2] << ", " << f[3] << "));\n";
                }
                o << "          } }\n";
                o << "      }\n";
                break;
            }
            case TP_MOV: case TP_BIN: case TP_BINS: case TP_EXP: case TP_RSQRT: {
                const TPSlot& d = tp.slots[in.dst];
                const int nj = d.cols > 1 ? 4 * nq(d.cols) : 1;
                if (in.op == TP_BINS) {
                    const bool fw = d.word == W_F32;
                    if (in.scalar_src >= 0) {
                        o << "      const unsigned long long raw = (unsigned long long)rec[b.nparams + b.naxis + " << in.scalar_src
                          << "];\n";
                        const int st = tp.scalar_types[in.scalar_src];
                        if (st == 0) o << (fw ? "      const unsigned ws = (unsigned)raw;\n"
                                              : "      const unsigned ws = (unsigned)(int)__uint_as_float((unsigned)raw);\n");
                        else if (st == 2) o << (fw ? "      const unsigned ws = __float_as_uint((float)(long long)raw);\n"
                                                   : "      const unsigned ws = (unsigned)(int)raw;\n");
                        else o << (fw ? "      const unsigned ws = __float_as_uint((float)(int)raw);\n"
                                      : "      const unsigned ws = (unsigned)(int)raw;\n");
                    } else {
                        unsigned fbits;
                        std::memcpy(&fbits, &in.fval, 4);
                        o << "      const unsigned ws = "
                          << (fw ? std::to_string(fbits) + "u" : "(unsigned)(" + std::to_string(in.ival) + ")") << ";\n";
                    }
                }
                o << "      #pragma unroll\n      for (int j = 0; j < " << nj << "; ++j) {\n";
                std::string rhs;
                const std::string a = elem(in.a, "j");
                if (in.op == TP_MOV) rhs = a;
                else if (in.op == TP_BIN) rhs = bin_expr(d.word, in.sub, a, in.mode == MODE_ROW ? elem(in.b, "0") : elem(in.b, "j"));
                else if (in.op == TP_BINS) rhs = in.scalar_first ? bin_expr(d.word, in.sub, "ws", a) : bin_expr(d.word, in.sub, a, "ws");
                else if (in.op == TP_EXP) rhs = "__float_as_uint(expf(__uint_as_float(" + a + ")))";
                else rhs = "__float_as_uint(__fdiv_rn(1.0f, sqrtf(__uint_as_float(" + a + "))))";
                o << "        " << elem(in.dst, "j") << " = " << rhs << ";\n";
                o << "      }\n";
                break;
            }
            case TP_ROWSUM: case TP_ROWMAX: case TP_ROWMEAN: {
                const TPSlot& a = tp.slots[in.a];
                const bool mx = in.op == TP_ROWMAX;
                o << "      float acc = " << (mx ? "-__int_as_float(0x7f800000)" : "0.f") << ";\n";
                if (a.cols > 1) {
                    o << "      #pragma unroll\n      for (int j = 0; j < " << 4 * nq(a.cols) << "; ++j)\n";
                    o << "        if ((j >> 2) < " << a.cols / (4 * L) << " || 4 * (sub + " << L << " * (j >> 2)) < " << a.cols << ") acc = "
                      << (mx ? "fmaxf(acc, __uint_as_float(" + elem(in.a, "j") + "))"
                             : "__fadd_rn(acc, __uint_as_float(" + elem(in.a, "j") + "))")
                      << ";\n";
                } else {
                    o << "      if (sub == 0) acc = __uint_as_float(" << elem(in.a, "0") << ");\n";
                }
                if (L > 1)
                    o << "      #pragma unroll\n      for (int o = " << L / 2 << "; o > 0; o >>= 1) acc = "
                      << (mx ? "fmaxf(acc, __shfl_xor_sync(0xffffffffu, acc, o))" : "__fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o))")
                      << ";\n";
                if (in.op == TP_ROWMEAN) o << "      acc = __fdiv_rn(acc, (float)" << in.k << ");\n";
                o << "      " << elem(in.dst, "0") << " = __float_as_uint(acc);\n";
                break;
            }
            default: break;
        }
        o << "    }\n";
    }
    o << "  }\n}\n";
}

}  // namespace

bool vector_form(const TileProgram& tp_in, const int* param_types) {
    const TileProgram tp = normalize(tp_in);
    for (int ii = 0; ii < tp.ninstr; ++ii) {
        const TPInstr& in = tp.ins[ii];
        if (in.op != TP_LOAD && in.op != TP_STORE) continue;
        const TPSlot& t = tp.slots[in.op == TP_LOAD ? in.dst : in.a];
        const int pt = param_types[in.param];
        if (t.cols > 1 && (t.cols % 4 != 0 || !(pt == PT_F32 || pt == PT_I32 || pt == PT_U32 || pt == PT_F16))) return false;
    }
    return true;
}

std::string gen_row_kernel(const TileProgram& tp_in, const int* param_types, const std::string& name) {
    const TileProgram tp = normalize(tp_in);
    std::ostringstream o;
    o << "#define MAXP " << kMaxParams << "\n" << kPrelude;
    emit_row_kernel(o, tp, param_types, name);
    if (vector_form(tp, param_types)) emit_group_kernel(o, tp, param_types, name + "_v");
    return o.str();
}

namespace {
// Process-wide caches: a generated source is compiled once, and a cubin is loaded once per device, however many
// programs use it (programs built from the same plan generate the same sources).
std::mutex g_cache_mu;
std::unordered_map<std::string, std::string> g_cubins;  // name + '\0' + source -> cubin
std::unordered_map<std::string, CUmodule> g_modules;    // device + ':' + cubin -> module (lives until exit)
}  // namespace

bool compile_cubin(const std::string& src, const std::string& name, std::string* cubin, std::string* log) {
    const std::string key = name + '\0' + src;
    {
        std::lock_guard<std::mutex> g(g_cache_mu);
        auto it = g_cubins.find(key);
        if (it != g_cubins.end()) {
            *cubin = it->second;
            return true;
        }
    }
    const Nvrtc& n = nvrtc();
    if (!n.ok) {
        *log = "NVRTC not found";
        return false;
    }
    nvrtcProgram_t prog = nullptr;
    if (n.create(&prog, src.c_str(), (name + ".cu").c_str(), 0, nullptr, nullptr) != 0) {
        *log = "nvrtcCreateProgram failed";
        return false;
    }
    const char* opts[] = {"--gpu-architecture=sm_100a", "--std=c++17", "-default-device"};
    const int rc = n.compile(prog, 3, opts);
    size_t ls = 0;
    n.log_size(prog, &ls);
    if (ls > 1) {
        log->resize(ls);
        n.log(prog, log->data());
    }
    bool ok = rc == 0;
    if (ok) {
        size_t cs = 0;
        ok = n.cubin_size(prog, &cs) == 0 && cs > 0;
        if (ok) {
            cubin->resize(cs);
            ok = n.cubin(prog, cubin->data()) == 0;
        }
    }
    n.destroy(&prog);
    if (!ok && log->empty()) *log = "NVRTC compilation failed";
    if (ok) {
        std::lock_guard<std::mutex> g(g_cache_mu);
        g_cubins.emplace(key, *cubin);
    }
    return ok;
}

bool load_cubin(const std::string& cubin, const std::string& name, void** fn, std::string* log) {
    const Driver& d = driver();
    if (!d.ok) {
        *log = "driver entry points unavailable";
        return false;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) {
        *log = "no current device";
        return false;
    }
    CUfunction f = nullptr;
    std::lock_guard<std::mutex> g(g_cache_mu);
    const std::string key = std::to_string(dev) + ':' + cubin;
    auto it = g_modules.find(key);
    if (it == g_modules.end()) {
        CUmodule mod = nullptr;  // kept for the life of the process: kernels of any program may run until exit
        if (d.load(&mod, cubin.data()) != CUDA_SUCCESS) {
            *log = "module load failed";
            return false;
        }
        it = g_modules.emplace(key, mod).first;
    }
    if (d.get(&f, it->second, name.c_str()) != CUDA_SUCCESS) {
        *log = "kernel '" + name + "' not in the module";
        return false;
    }
    *fn = reinterpret_cast<void*>(f);
    return true;
}

cudaError_t launch_row_kernel(void* fn, const TaskBatch& b, int rows, int workers, cudaStream_t s) {
    const Driver& d = driver();
    const int64_t nrows = b.ntasks * rows;
    int64_t blocks = std::min<int64_t>((nrows + 7) / 8, static_cast<int64_t>(sm_count()) * 8);  // 8 warps per block
    if (workers > 0) blocks = std::min<int64_t>(blocks, workers);
    blocks = std::max<int64_t>(blocks, 1);
    TaskBatch tb = b;
    void* args[] = {&tb};
    const CUresult r = d.launch(reinterpret_cast<CUfunction>(fn), static_cast<unsigned>(blocks), 1, 1, 256, 1, 1, 0,
                                reinterpret_cast<CUstream>(s), args, nullptr);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorLaunchFailure;
}

}  // namespace ptowsp::jit
