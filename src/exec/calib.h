// Init-time path calibration: measures, on the clique's own GPUs and all at
// once, the SM-driven NVLink pull bandwidth, the copy-engine peer-copy
// bandwidth (alone and alongside SM pulls), the pinned-host PCIe bandwidth
// (D2H and H2D, every GPU concurrently) and the CPU fold throughput. Results
// (with the route tuning of abi/tune.cc) are optionally cached in a JSON
// file keyed by GPU UUIDs and driver version (NCCL_B200_CALIB_CACHE).
#pragma once

#include <string>

#include "core/calib_model.h"
#include "core/policy.h"
#include "core/summary.h"

namespace nb {

CalibResult calibrate(const int* devices, int n, const Policy& p, Summary* s);
std::string calib_cache_key(const int* devices, int n);
bool calib_load(const std::string& path, const std::string& key, CalibResult* out);
void calib_save(const std::string& path, const std::string& key, const CalibResult& c);

}  // namespace nb
