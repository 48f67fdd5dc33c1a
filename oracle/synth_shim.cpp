// synth_shim.cpp — TEST INFRASTRUCTURE. Lets the package's seeded synthetic-GGUF writer
// (csrc/synth.cpp, csrc/gguf.cpp) be built on its own into oracle/libsynth.so, so that the
// benchmark's CPU reference arm can write the same model file without loading the product library
// libfence_b200.so. It supplies the one library helper those two files call.
#include <cstdarg>
#include <cstdio>

namespace fence {
static thread_local char g_synth_msg[512];

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_synth_msg, sizeof g_synth_msg, fmt, ap);
    va_end(ap);
    return code;
}
}  // namespace fence

extern "C" const char* oracle_synth_last_error(void) { return fence::g_synth_msg; }
