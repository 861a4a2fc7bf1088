// The device status word shared by every kernel of the library (see common.cuh).
#include "common.cuh"

namespace ms {
__device__ int g_device_status = 0;
__device__ unsigned long long g_wait_limit_ns = kDefaultWaitLimitNs;
std::atomic<long long> g_host_launches{0};
std::atomic<int> g_pdl_enabled{1};
std::atomic<int> g_pair_tiles_enabled{0};
}  // namespace ms
