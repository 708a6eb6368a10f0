// pdl.cu -- the thread-local switch behind PdlScope (common.cuh).
#include <cuda_runtime.h>

#include "common.cuh"

namespace pyxis {
namespace {
thread_local bool g_pdl = false;
}
bool pdl_enabled() { return g_pdl; }
PdlScope::PdlScope() : prev(g_pdl) { g_pdl = true; }
PdlScope::~PdlScope() { g_pdl = prev; }
}  // namespace pyxis
