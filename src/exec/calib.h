// Init-time path calibration: measures, on the clique's own GPUs and all at
// once, the SM-driven NVLink pull bandwidth, the copy-engine peer-copy
// bandwidth (alone and alongside SM pulls), the pinned-host PCIe bandwidth
// (D2H and H2D, every GPU concurrently) and the CPU fold throughput. Results
// are optionally cached in a JSON file keyed by GPU UUIDs, driver and NCCL
// versions (NCCL_B200_CALIB_CACHE).
#pragma once

#include "core/calib_model.h"
#include "core/policy.h"
#include "core/summary.h"

namespace nb {

CalibResult calibrate(const int* devices, int n, const Policy& p, Summary* s);
const CalibResult& last_calibration();
// Calibrate (or load the cache) and return the AllReduce shares.
Shares calibrate_shares(const int* devices, int n, const Policy& p, Summary* s);

}  // namespace nb
