// Clean-room CPU stand-in for the subset of the pto-isa tile library that the reference's generated CPU-sim
// artifacts call (TEST / BASELINE INFRASTRUCTURE ONLY).
//
// pto-isa is a third-party dependency of the reference (an un-vendored git submodule,
// `.gitmodules:1-3` -> https://gitcode.com/uvxiao/pto-isa.git, no commit pinned in the reference tree) and is
// absent here; no line of it was seen.  Every type and operation below is written from how the reference's own
// code uses it -- the wrappers in include/pto/wsp/codegen/abi/ptoisa_bridge.hpp:67-303, the kernels the emitter
// writes (src/python/pto_codegen.cpp:470-1241) and the example kernel bodies -- and from what the reference's
// checks demand of the results (numpy goldens of examples/*/golden.py; the top-k tie rule of
// examples/deepseek_lightning_indexer/golden.py:6-25).  Element semantics are those of this repository's numpy
// restatement of the same ops (oracle/cpu_sim.py), so the two oracles can be compared result for result:
//   * a tile's element (r, c) lives at data()[r * Cols + c] (Cols = the static, padded column count); ops work on
//     the valid region, GetValidRow() x GetValidCol();
//   * TLOAD / TSTORE copy the global view's shape (rows x cols at element strides s3, s4);
//   * f32 TMATMUL accumulates over k in order from zero with one fused multiply-add per step (f16 operands are
//     widened exactly); TROWSUM adds columns left to right; max / min propagate NaN like numpy;
//   * a row broadcast operand (TROWEXPAND*) gives element r to row r, whether it is stored as [R, 1] or [1, R];
//     a column broadcast operand (TCOLEXPAND*) gives element c to column c;
//   * TCVT rounds to nearest even; TSORT32 orders (score, index) pairs by score descending, ties in input order.
#pragma once

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <numeric>
#include <type_traits>
#include <vector>

using half = _Float16;  // IEEE binary16; emitted kernels name it unqualified

namespace pto {

constexpr int DYNAMIC = -1;

enum class TileType { Vec, Left, Right, Acc };
enum class BLayout { RowMajor, ColMajor };
enum class Layout { ND, DN, NZ };
enum class RoundMode { CAST_RINT, CAST_ROUND, CAST_FLOOR, CAST_CEIL, CAST_TRUNC, CAST_NONE };

template <TileType Kind, typename T, int R, int C, BLayout BL = BLayout::RowMajor, int VR = DYNAMIC, int VC = DYNAMIC>
class Tile {
   public:
    using DType = T;
    static constexpr int Rows = R;
    static constexpr int Cols = C;

    Tile() : Tile(static_cast<size_t>(VR == DYNAMIC ? R : VR), static_cast<size_t>(VC == DYNAMIC ? C : VC)) {}
    Tile(size_t valid_rows, size_t valid_cols)
        : buf_(static_cast<size_t>(R) * C, T{}), vr_(static_cast<int>(valid_rows)), vc_(static_cast<int>(valid_cols)) {}

    T* data() { return buf_.data(); }
    const T* data() const { return buf_.data(); }
    int GetValidRow() const { return vr_; }
    int GetValidCol() const { return vc_; }
    T& at(int r, int c) { return buf_[static_cast<size_t>(r) * C + c]; }
    const T& at(int r, int c) const { return buf_[static_cast<size_t>(r) * C + c]; }

   private:
    std::vector<T> buf_;  // on the heap: contraction tiles reach hundreds of KB
    int vr_, vc_;
};

template <typename T, int R, int C, int VR = DYNAMIC, int VC = DYNAMIC>
using TileLeft = Tile<TileType::Left, T, R, C, BLayout::RowMajor, VR, VC>;
template <typename T, int R, int C, int VR = DYNAMIC, int VC = DYNAMIC>
using TileRight = Tile<TileType::Right, T, R, C, BLayout::RowMajor, VR, VC>;
template <typename T, int R, int C, int VR = DYNAMIC, int VC = DYNAMIC>
using TileAcc = Tile<TileType::Acc, T, R, C, BLayout::RowMajor, VR, VC>;

// Global views: the emitted code uses 5-D shapes/strides of which only the last two are dynamic.
template <int D0, int D1, int D2, int D3, int D4>
struct Shape {
    int rows = D3, cols = D4;
    Shape() = default;
    Shape(int r, int c) : rows(r), cols(c) {}
};
template <int S0, int S1, int S2, int S3, int S4>
struct Stride {
    int64_t s3 = S3, s4 = S4;
    Stride() = default;
    Stride(int64_t a, int64_t b) : s3(a), s4(b) {}
};
template <typename T, typename ShapeT, typename StrideT, Layout L = Layout::ND>
struct GlobalTensor {
    T* ptr;
    ShapeT shape;
    StrideT stride;
    GlobalTensor(T* p, ShapeT sh, StrideT st) : ptr(p), shape(sh), stride(st) {}
};

namespace detail {

template <typename T>
inline float widen(T x) {
    return static_cast<float>(x);
}

template <typename Dst, typename Src>
inline Dst narrow(Src x) {
    return static_cast<Dst>(x);  // _Float16 conversion rounds to nearest even
}

template <typename T>
inline T nan_max(T a, T b) {
    if (std::isnan(static_cast<double>(a))) return a;
    if (std::isnan(static_cast<double>(b))) return b;
    return a < b ? b : a;
}
template <typename T>
inline T nan_min(T a, T b) {
    if (std::isnan(static_cast<double>(a))) return a;
    if (std::isnan(static_cast<double>(b))) return b;
    return b < a ? b : a;
}

// Element `i` of a broadcast vector stored either as one column ([n, 1]) or one row ([1, n]).
template <typename TileT>
inline auto vec_at(const TileT& t, int i) {
    return t.GetValidCol() == 1 && t.GetValidRow() > 1 ? t.at(i, 0) : t.at(0, i);
}

template <typename TD, typename TA, typename TB, typename F>
inline int elementwise(TD& d, TA& a, TB& b, F f) {
    using T = typename TD::DType;
    for (int r = 0; r < d.GetValidRow(); ++r)
        for (int c = 0; c < d.GetValidCol(); ++c) d.at(r, c) = static_cast<T>(f(a.at(r, c), b.at(r, c)));
    return 0;
}
template <typename TD, typename TA, typename TB, typename F>
inline int row_expand(TD& d, TA& a, TB& b, F f) {
    using T = typename TD::DType;
    for (int r = 0; r < d.GetValidRow(); ++r) {
        const auto s = vec_at(b, r);
        for (int c = 0; c < d.GetValidCol(); ++c) d.at(r, c) = static_cast<T>(f(a.at(r, c), s));
    }
    return 0;
}
template <typename TD, typename TA, typename TB, typename F>
inline int col_expand(TD& d, TA& a, TB& b, F f) {
    using T = typename TD::DType;
    for (int r = 0; r < d.GetValidRow(); ++r)
        for (int c = 0; c < d.GetValidCol(); ++c) d.at(r, c) = static_cast<T>(f(a.at(r, c), vec_at(b, c)));
    return 0;
}
template <typename TD, typename TS, typename F>
inline int unary(TD& d, TS& s, F f) {
    using T = typename TD::DType;
    for (int r = 0; r < d.GetValidRow(); ++r)
        for (int c = 0; c < d.GetValidCol(); ++c) d.at(r, c) = static_cast<T>(f(s.at(r, c)));
    return 0;
}

}  // namespace detail

// ---- data movement ----------------------------------------------------------------------------------------------

template <typename TileT, typename GT, typename... E>
inline int TLOAD(TileT& dst, GT& src, E&...) {
    using T = typename TileT::DType;
    for (int r = 0; r < src.shape.rows; ++r)
        for (int c = 0; c < src.shape.cols; ++c)
            dst.at(r, c) = static_cast<T>(src.ptr[r * src.stride.s3 + c * src.stride.s4]);
    return 0;
}

template <typename GT, typename TileT, typename... E>
inline int TSTORE(GT& dst, TileT& src, E&...) {
    using T = std::remove_cv_t<std::remove_pointer_t<decltype(dst.ptr)>>;
    for (int r = 0; r < dst.shape.rows; ++r)
        for (int c = 0; c < dst.shape.cols; ++c)
            dst.ptr[r * dst.stride.s3 + c * dst.stride.s4] = static_cast<T>(src.at(r, c));
    return 0;
}

template <typename TD, typename TS>
inline int TMOV(TD& dst, TS& src) {
    return detail::unary(dst, src, [](auto x) { return x; });
}

template <typename TD, typename TS, typename... Rest>
inline int TCVT(TD& dst, TS& src, Rest&&...) {
    using T = typename TD::DType;
    return detail::unary(dst, src, [](auto x) { return detail::narrow<T>(x); });
}

// ---- contraction ------------------------------------------------------------------------------------------------

template <typename TC, typename TA, typename TB, typename... E>
inline int TMATMUL(TC& c, TA& a, TB& b, E&...) {
    const int M = a.GetValidRow(), K = a.GetValidCol(), N = b.GetValidCol();
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) {
            float acc = 0.f;
            for (int k = 0; k < K; ++k) acc = std::fma(detail::widen(a.at(i, k)), detail::widen(b.at(k, j)), acc);
            c.at(i, j) = static_cast<typename TC::DType>(acc);
        }
    return 0;
}

// ---- element-wise -----------------------------------------------------------------------------------------------

#define PTOWSP_STANDIN_BINARY(NAME, EXPR)                                             \
    template <typename TD, typename TA, typename TB, typename... E>                    \
    inline int NAME(TD& d, TA& a, TB& b, E&...) {                                       \
        return detail::elementwise(d, a, b, [](auto x, auto y) { return EXPR; });      \
    }
PTOWSP_STANDIN_BINARY(TADD, x + y)
PTOWSP_STANDIN_BINARY(TSUB, x - y)
PTOWSP_STANDIN_BINARY(TMUL, x* y)
PTOWSP_STANDIN_BINARY(TDIV, x / y)
PTOWSP_STANDIN_BINARY(TMAX, detail::nan_max(x, y))
PTOWSP_STANDIN_BINARY(TMIN, detail::nan_min(x, y))
#undef PTOWSP_STANDIN_BINARY

#define PTOWSP_STANDIN_ROWEXPAND(NAME, EXPR)                                          \
    template <typename TD, typename TA, typename TB, typename... E>                    \
    inline int NAME(TD& d, TA& a, TB& b, E&...) {                                       \
        return detail::row_expand(d, a, b, [](auto x, auto y) { return EXPR; });       \
    }
PTOWSP_STANDIN_ROWEXPAND(TROWEXPANDADD, x + y)
PTOWSP_STANDIN_ROWEXPAND(TROWEXPANDSUB, x - y)
PTOWSP_STANDIN_ROWEXPAND(TROWEXPANDMUL, x* y)
PTOWSP_STANDIN_ROWEXPAND(TROWEXPANDDIV, x / y)
PTOWSP_STANDIN_ROWEXPAND(TROWEXPANDMAX, detail::nan_max(x, y))
PTOWSP_STANDIN_ROWEXPAND(TROWEXPANDMIN, detail::nan_min(x, y))
#undef PTOWSP_STANDIN_ROWEXPAND

#define PTOWSP_STANDIN_COLEXPAND(NAME, EXPR)                                          \
    template <typename TD, typename TA, typename TB, typename... E>                    \
    inline int NAME(TD& d, TA& a, TB& b, E&...) {                                       \
        return detail::col_expand(d, a, b, [](auto x, auto y) { return EXPR; });       \
    }
PTOWSP_STANDIN_COLEXPAND(TCOLEXPANDSUB, x - y)
PTOWSP_STANDIN_COLEXPAND(TCOLEXPANDMUL, x* y)
PTOWSP_STANDIN_COLEXPAND(TCOLEXPANDDIV, x / y)
#undef PTOWSP_STANDIN_COLEXPAND

// Tile-and-scalar forms; TDIVS also takes the scalar first (scalar / tile).
template <typename TD, typename TS, typename S>
inline int TADDS(TD& d, TS& s, S v) {
    using T = typename TD::DType;
    return detail::unary(d, s, [v](auto x) { return x + static_cast<T>(v); });
}
template <typename TD, typename TS, typename S>
inline int TSUBS(TD& d, TS& s, S v) {
    using T = typename TD::DType;
    return detail::unary(d, s, [v](auto x) { return x - static_cast<T>(v); });
}
template <typename TD, typename TS, typename S>
inline int TMULS(TD& d, TS& s, S v) {
    using T = typename TD::DType;
    return detail::unary(d, s, [v](auto x) { return x * static_cast<T>(v); });
}
template <typename TD, typename TS, typename S, std::enable_if_t<!std::is_arithmetic_v<TS>, int> = 0>
inline int TDIVS(TD& d, TS& s, S v) {
    using T = typename TD::DType;
    return detail::unary(d, s, [v](auto x) { return x / static_cast<T>(v); });
}
template <typename TD, typename S, typename TS, std::enable_if_t<std::is_arithmetic_v<S>, int> = 0>
inline int TDIVS(TD& d, S v, TS& s) {
    using T = typename TD::DType;
    return detail::unary(d, s, [v](auto x) { return static_cast<T>(v) / x; });
}
template <typename TD, typename TS, typename S>
inline int TMAXS(TD& d, TS& s, S v) {
    using T = typename TD::DType;
    return detail::unary(d, s, [v](auto x) { return detail::nan_max(x, static_cast<T>(v)); });
}
template <typename TD, typename TS, typename S>
inline int TMINS(TD& d, TS& s, S v) {
    using T = typename TD::DType;
    return detail::unary(d, s, [v](auto x) { return detail::nan_min(x, static_cast<T>(v)); });
}

template <typename TD, typename TS>
inline int TEXP(TD& d, TS& s) {
    return detail::unary(d, s, [](auto x) { return std::exp(detail::widen(x)); });
}
template <typename TD, typename TS>
inline int TRSQRT(TD& d, TS& s) {
    return detail::unary(d, s, [](auto x) { return 1.0f / std::sqrt(detail::widen(x)); });
}

// ---- row reductions ([R, C] -> [R, 1]); the scratch tile is not needed here (it may alias the source) ----------

template <typename TD, typename TS, typename TT>
inline int TROWSUM(TD& d, TS& s, TT&) {
    using T = typename TD::DType;
    std::vector<T> out(static_cast<size_t>(s.GetValidRow()));
    for (int r = 0; r < s.GetValidRow(); ++r) {
        T acc = T{};
        for (int c = 0; c < s.GetValidCol(); ++c) acc = static_cast<T>(acc + s.at(r, c));
        out[r] = acc;
    }
    for (int r = 0; r < s.GetValidRow(); ++r) d.at(r, 0) = out[r];
    return 0;
}
template <typename TD, typename TS, typename TT>
inline int TROWMAX(TD& d, TS& s, TT&) {
    using T = typename TD::DType;
    std::vector<T> out(static_cast<size_t>(s.GetValidRow()));
    for (int r = 0; r < s.GetValidRow(); ++r) {
        T m = static_cast<T>(s.at(r, 0));
        for (int c = 1; c < s.GetValidCol(); ++c) m = detail::nan_max(m, static_cast<T>(s.at(r, c)));
        out[r] = m;
    }
    for (int r = 0; r < s.GetValidRow(); ++r) d.at(r, 0) = out[r];
    return 0;
}

// ---- sort: (score, index) pairs, score descending, ties in input order ------------------------------------------

template <typename TD, typename TS, typename TI, typename... Tmp>
inline int TSORT32(TD& d, TS& s, TI& idx, Tmp&...) {
    const int vc = s.GetValidCol(), n = s.GetValidRow() * vc;  // the valid region in row-major order
    std::vector<int> order(static_cast<size_t>(n));
    std::iota(order.begin(), order.end(), 0);
    auto score = [&](int i) { return detail::widen(s.at(i / vc, i % vc)); };
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return score(x) > score(y); });
    using T = typename TD::DType;
    for (int i = 0; i < n; ++i) {
        d.data()[2 * i] = static_cast<T>(score(order[i]));
        d.data()[2 * i + 1] = static_cast<T>(idx.at(order[i] / vc, order[i] % vc));
    }
    return 0;
}

}  // namespace pto
