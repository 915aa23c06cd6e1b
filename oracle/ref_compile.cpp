// Artifact builder for the reference CPU-sim (TEST / BASELINE INFRASTRUCTURE ONLY).
//
// The reference compiles each generated CPU-sim artifact (workload_main.cpp + one kernel_<name>.cpp per kernel)
// through a generated CMake project (src/pto/wsp/codegen/cmake_compiler.cpp:175-270).  This file is linked into
// oracle/_ref's build of the reference IR module in place of that one: same entry point
// (include/pto/wsp/codegen/cmake_compiler.hpp), same inputs and result, but the sources are compiled by one direct
// g++ call -- no CMake -- with the same definitions the reference's project sets (C++23, -O3, __CPU_SIM=1, position
// independent), against the reference's own ABI headers and this repository's clean-room pto-isa stand-in
// (oracle/ptoisa/pto/pto-inst.hpp).  Artifacts are cached by a hash of their sources under PTOWSP_ARTIFACT_DIR
// (default: the directory given at build time).
#include <cstdint>
#include <cstdlib>
#include <filesystem>
#include <fstream>
#include <map>
#include <sstream>
#include <stdexcept>
#include <string>

#include "pto/wsp/codegen/cmake_compiler.hpp"

#ifndef PTOWSP_REF_INCLUDE
#error "build with -DPTOWSP_REF_INCLUDE=\"<reference>/include\""
#endif
#ifndef PTOWSP_PTOISA_INCLUDE
#error "build with -DPTOWSP_PTOISA_INCLUDE=\"<this repo>/oracle/ptoisa\""
#endif
#ifndef PTOWSP_ARTIFACT_DEFAULT
#error "build with -DPTOWSP_ARTIFACT_DEFAULT=\"<dir>\""
#endif

namespace fs = std::filesystem;

namespace pto::wsp::codegen {
namespace {

uint64_t fnv(uint64_t h, const std::string& s) {
    for (unsigned char c : s) {
        h ^= c;
        h *= 1099511628211ull;
    }
    return h;
}

std::string slurp(const fs::path& p) {
    std::ifstream f(p, std::ios::binary);
    std::ostringstream o;
    o << f.rdbuf();
    return o.str();
}

std::string quote(const std::string& s) {
    std::string o = "'";
    for (char c : s) o += (c == '\'') ? std::string("'\\''") : std::string(1, c);
    return o + "'";
}

}  // namespace

CompileResult compile_sources_via_cmake(const std::map<std::string, std::string>& sources,
                                        const std::string& output_name) {
    if (sources.empty()) throw std::runtime_error("compile_sources_via_cmake: no sources provided");
    const char* env = std::getenv("PTOWSP_ARTIFACT_DIR");
    const fs::path root = env && *env ? fs::path(env) : fs::path(PTOWSP_ARTIFACT_DEFAULT);
    const char* cxx_env = std::getenv("PTOWSP_ARTIFACT_CXX");
    const std::string cxx = cxx_env && *cxx_env ? cxx_env : "/usr/bin/g++";
    uint64_t h = 1469598103934665603ull;
    for (const auto& [name, content] : sources) h = fnv(fnv(h, name), content);
    h = fnv(h, slurp(fs::path(PTOWSP_PTOISA_INCLUDE) / "pto" / "pto-inst.hpp"));
    char key[17];
    std::snprintf(key, sizeof key, "%016llx", static_cast<unsigned long long>(h));
    const fs::path so = root / (output_name + "_" + key + ".so");
    if (fs::exists(so)) return CompileResult{so.string(), key};
    const fs::path src = root / ("src_" + output_name + "_" + key);
    fs::create_directories(src);
    std::string files;
    for (const auto& [name, content] : sources) {
        const fs::path p = src / name;
        fs::create_directories(p.parent_path());
        std::ofstream(p, std::ios::binary) << content;
        if (p.extension() == ".cpp") files += " " + quote(p.string());
    }
    const fs::path tmp = root / (output_name + "_" + key + ".so.tmp");
    const std::string cmd = quote(cxx) + " -std=c++23 -O3 -fPIC -shared -D__CPU_SIM=1 -Wno-deprecated-declarations" +
                            " -I" + quote(PTOWSP_REF_INCLUDE) + " -I" + quote(PTOWSP_PTOISA_INCLUDE) + files +
                            " -o " + quote(tmp.string()) + " > " + quote((src / "build.log").string()) + " 2>&1";
    if (std::system(cmd.c_str()) != 0)
        throw std::runtime_error("CPU-sim artifact build failed. See " + (src / "build.log").string());
    fs::rename(tmp, so);
    return CompileResult{so.string(), key};
}

}  // namespace pto::wsp::codegen
