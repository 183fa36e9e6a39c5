// TEST INFRASTRUCTURE ONLY. Minimal stand-in for the glog logging macros that
// the reference sources use (CHECK*, LOG(level)); it carries no arithmetic. It
// lets oracle/Makefile compile the reference's own kernel sources in place.
#pragma once
#include <cstdio>
#include <cstdlib>
#include <sstream>
#include <string>
// glog's header pulls these in transitively; the reference relies on that.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <vector>

namespace fire_ref_shim {
struct Sink {
    bool fatal;
    const char* file;
    int line;
    std::ostringstream os;
    Sink(bool f, const char* fl, int ln) : fatal(f), file(fl), line(ln) {}
    ~Sink() {
        if (fatal) {
            std::fprintf(stderr, "[ref FATAL %s:%d] %s\n", file, line, os.str().c_str());
            std::abort();
        }
    }
    template <typename T> Sink& operator<<(const T& v) { os << v; return *this; }
};
struct Voidify { void operator&(Sink&) {} };
}  // namespace fire_ref_shim

#define FIRE_REF_SINK(fatal) fire_ref_shim::Sink((fatal), __FILE__, __LINE__)
#define LOG(level) FIRE_REF_SINK(std::string(#level) == "FATAL")
#define CHECK(cond) (cond) ? (void)0 : fire_ref_shim::Voidify() & FIRE_REF_SINK(true) << "Check failed: " #cond " "
#define CHECK_OP(a, b, op) CHECK((a) op (b))
#define CHECK_EQ(a, b) CHECK_OP(a, b, ==)
#define CHECK_NE(a, b) CHECK_OP(a, b, !=)
#define CHECK_GT(a, b) CHECK_OP(a, b, >)
#define CHECK_GE(a, b) CHECK_OP(a, b, >=)
#define CHECK_LT(a, b) CHECK_OP(a, b, <)
#define CHECK_LE(a, b) CHECK_OP(a, b, <=)
