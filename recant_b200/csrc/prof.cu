// Optional launch profiler: when enabled, every kernel launch of the library is bracketed by a
// pair of CUDA events recorded on the launching stream, so a caller can attribute device time
// to kernels without an external profiler. Disabled by default; not thread-safe (one driver
// thread, as in a benchmark).
#include <cstring>
#include <vector>

#include "common.cuh"

namespace rb2 {

namespace {
struct Slot {
  const char* name;
  cudaEvent_t a, b;
};
bool g_on = false;
std::vector<Slot> g_slots;
size_t g_used = 0;
size_t g_dropped = 0;
}  // namespace

ProfScope::ProfScope(const char* name, cudaStream_t s) : slot_(-1), s_(s) {
  if (!g_on) return;
  if (g_used >= g_slots.size()) { ++g_dropped; return; }
  slot_ = int(g_used++);
  g_slots[slot_].name = name;
  cudaEventRecord(g_slots[slot_].a, s);
}

ProfScope::~ProfScope() {
  if (slot_ >= 0) cudaEventRecord(g_slots[slot_].b, s_);
}

}  // namespace rb2

using namespace rb2;

extern "C" int rb2_profile_enable(int max_launches) {
  RB2_CHECK_ARG(max_launches > 0 && max_launches <= (1 << 20), "profile_enable: bad capacity");
  if (int(g_slots.size()) < max_launches) {
    size_t old = g_slots.size();
    g_slots.resize(max_launches);
    for (size_t i = old; i < g_slots.size(); ++i) {
      RB2_CUDA(cudaEventCreate(&g_slots[i].a), "profile_enable");
      RB2_CUDA(cudaEventCreate(&g_slots[i].b), "profile_enable");
    }
  }
  g_used = 0;
  g_dropped = 0;
  g_on = true;
  return RB2_OK;
}

extern "C" int rb2_profile_disable(void) {
  g_on = false;
  return RB2_OK;
}

extern "C" int rb2_profile_read(int max_records, char* names, size_t name_stride, float* ms) {
  // waits for the recorded events; returns the number of records (or -1 on error)
  const size_t n = g_used < size_t(max_records) ? g_used : size_t(max_records);
  for (size_t i = 0; i < n; ++i) {
    if (cudaEventSynchronize(g_slots[i].b) != cudaSuccess) { set_error("profile_read: sync failed"); return -1; }
    float t = 0.f;
    if (cudaEventElapsedTime(&t, g_slots[i].a, g_slots[i].b) != cudaSuccess) { set_error("profile_read: elapsed"); return -1; }
    ms[i] = t;
    std::strncpy(names + i * name_stride, g_slots[i].name, name_stride - 1);
    names[i * name_stride + name_stride - 1] = '\0';
  }
  return int(n);
}

extern "C" int rb2_profile_dropped(void) { return int(g_dropped); }
