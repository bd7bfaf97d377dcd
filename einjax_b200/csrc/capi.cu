// Library-wide entry points: version, launch counter, status strings.
#include "common.cuh"

namespace es {
std::atomic<int64_t> g_launches{0};
}

extern "C" int es_version(void) { return 100; }

extern "C" int64_t es_launch_count(void) { return es::g_launches.load(std::memory_order_relaxed); }

extern "C" void es_launch_count_reset(void) { es::g_launches.store(0, std::memory_order_relaxed); }

extern "C" const char* es_status_string(int status) {
  switch (status) {
    case ES_OK: return "ok";
    case ES_ERR_INVALID: return "invalid argument";
    case ES_ERR_INDEX: return "tile coordinate outside its grid";
    case ES_ERR_WORKSPACE: return "workspace too small";
    case ES_ERR_CUDA: return "CUDA error";
    case ES_ERR_UNSUPPORTED: return "unsupported dtype, rank or size";
    case ES_ERR_TIMEOUT: return "a bounded device-side wait ran out";
    default: return "unknown status";
  }
}
