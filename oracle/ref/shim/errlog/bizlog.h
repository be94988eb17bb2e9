// Logging stand-in used ONLY when oracle/Makefile compiles the reference's
// CPU quant sources into oracle/_ref/ (a test checker, never shipped).
//
// The reference's own errlog/bizlog.h needs spdlog + nlohmann_json, which
// are not installed here.  Its CPU quant path only *logs* through BIZLOG and
// never throws, so a macro that prints the numeric error code to stderr
// keeps the arithmetic under test identical.
#ifndef MLQ_ORACLE_REF_SHIM_BIZLOG_H_
#define MLQ_ORACLE_REF_SHIM_BIZLOG_H_

#include <cstdio>
#include <string>

#include <spdlog/spdlog.h>  // src/tensor.cc prints through spdlog directly

#include "generated/error_code_enum.h"

namespace mlq_ref_shim {
template <typename... Args>
inline void report(int code, const char* file, int line, Args&&...) {
    std::fprintf(stderr, "[reference errlog] code=%d at %s:%d\n", code, file, line);
}
}  // namespace mlq_ref_shim

#define BIZLOG(ec, ...) ::mlq_ref_shim::report(static_cast<int>(ec), __FILE__, __LINE__, ##__VA_ARGS__)
#define BIZLOG_S(ec, session_id, ...) \
    ::mlq_ref_shim::report(static_cast<int>(ec), __FILE__, __LINE__, (session_id), ##__VA_ARGS__)

#endif  // MLQ_ORACLE_REF_SHIM_BIZLOG_H_
