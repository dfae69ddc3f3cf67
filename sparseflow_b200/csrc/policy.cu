// Process-wide path policy: the documented choices between kernel paths that
// callers (and the parity tests, which force each path in turn) may make.
// Plain atomics; read on the host when a call plans its launch.
#include <atomic>
#include "policy.cuh"

namespace sf {
namespace {
std::atomic<long long> g_policy[SF_POLICY_COUNT] = {
    {0},    // SF_POLICY_CONV1X1_PATH: automatic
    {128},  // SF_POLICY_CONV1X1_TC_MIN_HW
    {0},    // SF_POLICY_CONV3X3_PATH: automatic
    {0},    // SF_POLICY_LIF_EVENTS_GENERAL
    {0},    // SF_POLICY_LIF_TC_EPILOGUE: automatic
};
}  // namespace

long long policy(int key) { return g_policy[key].load(std::memory_order_relaxed); }

}  // namespace sf

extern "C" sf_status sf_set_path_policy(int32_t key, int64_t value) {
  if (key < 0 || key >= SF_POLICY_COUNT || value < 0) return SF_ERR_INVALID_ARG;
  sf::g_policy[key].store(value, std::memory_order_relaxed);
  return SF_OK;
}

extern "C" int64_t sf_get_path_policy(int32_t key) {
  if (key < 0 || key >= SF_POLICY_COUNT) return -1;
  return sf::policy(key);
}
