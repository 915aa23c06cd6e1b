// Row-program compiler: row-local tile programs as fused CUDA kernels built with NVRTC (jit.cpp).
#pragma once

#include <cuda_runtime_api.h>

#include <string>

#include "device.hpp"

namespace ptowsp::jit {

// Whether every instruction of `tp` works on whole rows (loads/stores of full tiles, element-wise ops,
// row broadcasts, row reductions); otherwise `why` names the first obstacle.
bool row_local(const dev::TileProgram& tp, std::string* why);

// Rows of the program's tiles (one-row operands of column broadcasts aside).
int program_rows(const dev::TileProgram& tp);

// CUDA source of the fused kernel `name` for a row-local program; param_types[i] is the ParamType of param i.
// When vector_form() holds the source also has `name`_v, the variant with 16-byte (8-byte for f16) accesses
// for unit column strides and 16-byte-aligned rows.
std::string gen_row_kernel(const dev::TileProgram& tp, const int* param_types, const std::string& name);
bool vector_form(const dev::TileProgram& tp, const int* param_types);

// Compile `src` for sm_100a with NVRTC (no GPU needed); false with `log` set when NVRTC is unavailable or the
// compilation fails.
bool compile_cubin(const std::string& src, const std::string& name, std::string* cubin, std::string* log);

// Load kernel `name` of `cubin` into the current context.
bool load_cubin(const std::string& cubin, const std::string& name, void** fn, std::string* log);

// Launch a loaded row kernel over `b` (one warp per tile row of `rows` rows per task).
cudaError_t launch_row_kernel(void* fn, const dev::TaskBatch& b, int rows, int workers, cudaStream_t s);

}  // namespace ptowsp::jit
