#include "exec/calib.h"

#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <fstream>
#include <sstream>
#include <vector>

#include "core/hostreduce.h"
#include "exec/executor.h"
#include "kernels/kernels.h"

namespace nb {

namespace {

struct DevBufs {
  int dev = -1;
  void* a = nullptr;  // pulled from by the next device
  void* b = nullptr;  // destination of this device's pulls
  void* host = nullptr;
  size_t host_mapped = 0;
  cudaStream_t s1 = nullptr, s2 = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr, e2 = nullptr, e3 = nullptr;
};

bool ok(cudaError_t e) {
  if (e == cudaSuccess) return true;
  cudaGetLastError();
  return false;
}

}  // namespace

std::string calib_cache_key(const int* devices, int n) {
  std::ostringstream k;
  int drv = 0;
  cudaDriverGetVersion(&drv);
  k << "drv" << drv << "-n" << n;
  for (int i = 0; i < n; ++i) {
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, devices[i]) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    k << "-";
    for (int j = 0; j < 16; ++j) {
      char h[3];
      std::snprintf(h, sizeof h, "%02x", static_cast<unsigned char>(prop.uuid.bytes[j]));
      k << h;
    }
  }
  return k.str();
}

namespace {

// Time `body` on every device at once: each device's s1 records e0 before,
// and its streams record e1 (and e3 on s2) after; returns the max elapsed ms.
template <typename Body>
float time_all(std::vector<DevBufs>& d, Body body, bool use_s2) {
  for (auto& x : d) {
    if (!ok(cudaSetDevice(x.dev))) return -1;
    cudaDeviceSynchronize();
    cudaEventRecord(x.e0, x.s1);
    if (use_s2) cudaStreamWaitEvent(x.s2, x.e0, 0);
  }
  for (size_t i = 0; i < d.size(); ++i) {
    cudaSetDevice(d[i].dev);
    body(i);
  }
  float worst = 0;
  for (auto& x : d) {
    cudaSetDevice(x.dev);
    cudaEventRecord(x.e1, x.s1);
    if (use_s2) {
      cudaEventRecord(x.e3, x.s2);
      cudaStreamWaitEvent(x.s1, x.e3, 0);
      cudaEventRecord(x.e1, x.s1);
    }
  }
  for (auto& x : d) {
    cudaSetDevice(x.dev);
    if (!ok(cudaEventSynchronize(x.e1))) return -1;
    float ms = 0;
    if (!ok(cudaEventElapsedTime(&ms, x.e0, x.e1))) return -1;
    worst = std::max(worst, ms);
  }
  return worst;
}

}  // namespace

CalibResult calibrate(const int* devices, int n, const Policy& p, Summary* summary) {
  CalibResult r;
  if (n < 2) return r;
  const size_t bytes = 256 * kMiB, host_bytes = 64 * kMiB;
  std::vector<DevBufs> d(static_cast<size_t>(n));
  bool good = true;
  for (int i = 0; i < n && good; ++i) {
    DevBufs& x = d[size_t(i)];
    x.dev = devices[i];
    int target = -1, placed = -1;
    const char* method = "";
    good = ok(cudaSetDevice(x.dev)) && ok(cudaMalloc(&x.a, bytes)) && ok(cudaMalloc(&x.b, bytes)) &&
           ok(cudaMemset(x.a, 1, bytes)) &&
           ok(cudaStreamCreateWithFlags(&x.s1, cudaStreamNonBlocking)) &&
           ok(cudaStreamCreateWithFlags(&x.s2, cudaStreamNonBlocking)) &&
           ok(cudaEventCreate(&x.e0)) && ok(cudaEventCreate(&x.e1)) && ok(cudaEventCreate(&x.e2)) &&
           ok(cudaEventCreate(&x.e3));
    if (good) {
      x.host = alloc_pinned_near(x.dev, 2 * host_bytes, &x.host_mapped, &target, &placed, &method);
      good = x.host != nullptr;
    }
  }
  int sms = 0;
  if (good) good = ok(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, devices[0]));
  const LaunchShape shape = shape_for(bytes, sms, p.blocks_per_sm, p.threads);
  auto peer = [&](size_t i) -> DevBufs& { return d[(i + 1) % d.size()]; };
  const int reps = 3;
  if (good) {
    // SM pulls: device i copies device i+1's buffer into its own.
    float best = 1e30f;
    for (int k = 0; k < reps + 1; ++k) {
      const float ms = time_all(d, [&](size_t i) {
        CopyLaunch c;
        c.nseg = 1;
        c.src[0] = peer(i).a;
        c.dst[0] = d[i].b;
        c.len[0] = bytes;
        launch_copy(c, shape, d[i].s1);
      }, false);
      if (k && ms > 0) best = std::min(best, ms);
    }
    r.nvlink_sm_gbs = bytes / (best * 1e-3) / 1e9;
    // Copy engine alone.
    best = 1e30f;
    for (int k = 0; k < reps + 1; ++k) {
      const float ms = time_all(d, [&](size_t i) {
        cudaMemcpyAsync(d[i].b, peer(i).a, bytes, cudaMemcpyDefault, d[i].s1);
      }, false);
      if (k && ms > 0) best = std::min(best, ms);
    }
    r.nvlink_ce_gbs = bytes / (best * 1e-3) / 1e9;
    // SM and CE together on halves of the buffer, split by the CE's rate.
    const double f = r.nvlink_ce_gbs / (r.nvlink_ce_gbs + r.nvlink_sm_gbs);
    const size_t ce_part = (size_t(double(bytes) * f) / 16) * 16;
    best = 1e30f;
    for (int k = 0; k < reps + 1; ++k) {
      const float ms = time_all(d, [&](size_t i) {
        CopyLaunch c;
        c.nseg = 1;
        c.src[0] = static_cast<char*>(peer(i).a) + ce_part;
        c.dst[0] = static_cast<char*>(d[i].b) + ce_part;
        c.len[0] = bytes - ce_part;
        launch_copy(c, shape, d[i].s1);
        cudaMemcpyAsync(d[i].b, peer(i).a, ce_part, cudaMemcpyDefault, d[i].s2);
      }, true);
      if (k && ms > 0) best = std::min(best, ms);
    }
    r.nvlink_mix_gbs = bytes / (best * 1e-3) / 1e9;
    r.mix_ce_fraction = f;
    // PCIe: every GPU does D2H and H2D concurrently.
    best = 1e30f;
    for (int k = 0; k < reps + 1; ++k) {
      const float ms = time_all(d, [&](size_t i) {
        cudaMemcpyAsync(d[i].host, d[i].a, host_bytes, cudaMemcpyDeviceToHost, d[i].s1);
        cudaMemcpyAsync(d[i].b, static_cast<char*>(d[i].host) + host_bytes, host_bytes,
                        cudaMemcpyHostToDevice, d[i].s2);
      }, true);
      if (k && ms > 0) best = std::min(best, ms);
    }
    r.pcie_d2h_gbs = r.pcie_h2d_gbs = host_bytes / (best * 1e-3) / 1e9;
    // Host fold throughput over n sources (input bytes per second).
    std::vector<std::vector<float>> srcs(static_cast<size_t>(n), std::vector<float>(4 * kMiB, 1.0f));
    std::vector<float> out(4 * kMiB);
    const void* sp[kMaxRanks];
    for (int i = 0; i < n; ++i) sp[i] = srcs[size_t(i)].data();
    FoldParams fp;
    fp.dtype = DType::F32;
    fp.nranks = n;
    double best_s = 1e30;
    for (int k = 0; k < 3; ++k) {
      const auto t0 = std::chrono::steady_clock::now();
      host_fold_parallel(fp, sp, n, out.data(), out.size() * 4, p.host_threads);
      const double s = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
      best_s = std::min(best_s, s);
    }
    r.fold_gbs = double(n) * out.size() * 4 / best_s / 1e9;
    r.valid = r.nvlink_sm_gbs > 0;
  }
  for (auto& x : d) {
    if (x.dev < 0) continue;
    cudaSetDevice(x.dev);
    cudaDeviceSynchronize();
    if (x.a) cudaFree(x.a);
    if (x.b) cudaFree(x.b);
    if (x.host) free_pinned(x.host, 2 * host_bytes, x.host_mapped);
    for (cudaEvent_t e : {x.e0, x.e1, x.e2, x.e3})
      if (e) cudaEventDestroy(e);
    if (x.s1) cudaStreamDestroy(x.s1);
    if (x.s2) cudaStreamDestroy(x.s2);
  }
  cudaGetLastError();
  if (summary && r.valid) {
    char buf[320];
    std::snprintf(buf, sizeof buf,
                  "calibration nvlink_sm_gbs=%.1f nvlink_ce_gbs=%.1f nvlink_mix_gbs=%.1f "
                  "pcie_gbs=%.1f fold_gbs=%.1f",
                  r.nvlink_sm_gbs, r.nvlink_ce_gbs, r.nvlink_mix_gbs, r.pcie_h2d_gbs, r.fold_gbs);
    summary->note(buf);
  }
  return r;
}

bool calib_load(const std::string& path, const std::string& key, CalibResult* out) {
  if (path.empty()) return false;
  std::ifstream in(path);
  if (!in) return false;
  std::stringstream ss;
  ss << in.rdbuf();
  return calib_from_json(ss.str(), key, out);
}

void calib_save(const std::string& path, const std::string& key, const CalibResult& c) {
  if (path.empty() || !c.valid) return;
  std::ofstream out(path);
  if (out) out << calib_to_json(c, key);
}

}  // namespace nb
