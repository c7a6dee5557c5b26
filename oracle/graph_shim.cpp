// graph_shim.cpp -- TEST INFRASTRUCTURE ONLY.  Error plumbing for the host graph builder
// (graphgp.jl_b200/csrc/graph_build.cpp, a restatement of build_graph, src/graph_build.jl:256-288)
// when it is compiled into the oracle's own libgp_graph.so, so that bench.py's reference arm and
// the tests can build graphs without loading libgraphgp_b200.so.
#include <cstdarg>
#include <cstdio>

namespace gpb2 {

static thread_local char g_msg[512];

int set_error(int status, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return status;
}

void clear_error() { g_msg[0] = 0; }

}  // namespace gpb2

extern "C" const char* gpo_graph_last_error(void) { return gpb2::g_msg; }
