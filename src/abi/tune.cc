// Init-time route tuning: every candidate route of each collective runs on
// the clique's own GPUs (one warm-up and three timed runs on scratch
// buffers, CUDA events on every GPU, max over GPUs) and the fastest one is
// kept per collective kind. Candidates: AllReduce fused two-shot / staged /
// NVLS; ReduceScatter fused pull / staged; AllGather and Broadcast with SM or
// copy-engine data movement.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <string>
#include <vector>

#include "abi/runtime.h"
#include "core/plan.h"
#include "exec/nvls.h"

namespace nb {

namespace {

struct Candidate {
  Algo algo;
  int ce_ppm;
  int host_ppm;
  int piece_mib;  // staged routes
  int depth;
  int split_ppm = 0;     // hybrid routes: the switch's share (per 10000)
  int split_blocks = 0;  // and its blocks per GPU
  int nvls_shape = 0;    // NVLS routes: packed kernel shape (pack_nvls_shape)
};

// NVLS AllReduce kernel shapes tried (movers per block, requests in flight per
// mover, round MiB, round schedule): the switch side bounds the kernel, so
// more requests in flight may pay. No shape shrinks the round: the scratch
// holds one buffer per round of the largest message, and smaller rounds
// would reuse buffers within a call. The ramped schedule (NCCL_B200_NVLS_RAMP)
// measured no gain on 2 GPUs and is not a candidate. From four ranks the
// tuning also tries the copier that copies every round in first (the movers
// then never wait for a copy-in); on 2 GPUs it measured 2 % slower.
constexpr int kNvlsShapes[][5] = {{0, 0, 0, 0, 0}, {608, 4, 0, 0, 0}, {608, 8, 0, 0, 0}, {0, 0, 0, 0, 2},
                                  {608, 8, 0, 0, 2}};

// Every candidate route of a kind; a host-lane variant is added wherever the
// rate model (measured PCIe, NVLink and fold rates) predicts a host share.
std::vector<Candidate> candidates(Kind k, int n, bool nvls, const CalibResult& rates);

// Small messages: the routes whose every byte moves on the SMs, with no
// pipeline to start (one-shot and two-shot folds, pulls, pushes, NVLS).
std::vector<Candidate> tiny_candidates(Kind k, int n, bool nvls) {
  std::vector<Candidate> v;
  auto add = [&](Algo a) { v.push_back({a, 0, 0, 0, 0}); };
  switch (k) {
    case Kind::AllReduce:
      add(Algo::ArOneShot);
      add(Algo::ArTwoShotLL);
      add(Algo::ArTwoShot);
      if (nvls) add(Algo::ArNvls);
      break;
    case Kind::ReduceScatter:
      add(Algo::RsLL);
      add(Algo::RsPull);
      if (nvls) add(Algo::RsNvls);
      break;
    case Kind::AllGather:
      add(Algo::AgLL);
      add(Algo::AgPull);
      add(Algo::AgPush);
      if (nvls) add(Algo::AgNvls);
      break;
    case Kind::Broadcast:
      add(Algo::BcLL);
      add(n >= 3 ? Algo::BcScatter : Algo::BcPull);
      add(Algo::BcRing);
      if (nvls) add(Algo::BcNvls);
      break;
    default:
      break;
  }
  return v;
}

std::vector<Candidate> candidates(Kind k, int n, bool nvls, const CalibResult& rates) {
  std::vector<Candidate> v;
  auto add = [&](Algo a, int ce, int piece = 0, int depth = 0) {
    v.push_back({a, ce, 0, piece, depth});
    const int host = shares_from(rates, a, n).host_ppm;
    if (host > 0) v.push_back({a, ce, host, piece, depth});
  };
  // Copy-engine-staged and copy-engine-heavy variants only pay on two GPUs
  // (measured: at 4 and 8 ranks they trail the SM routes by 2-7x), so larger
  // cliques skip them and tune faster.
  const bool small = n <= 2;
  switch (k) {
    case Kind::AllReduce:
      add(Algo::ArTwoShot, 0);
      v.push_back({Algo::ArTwoShotLL, 0, 0, 0, 0});
      if (small) {
        add(Algo::ArStaged, 0, 64, 3);
        add(Algo::ArStaged, 0, 128, 2);
        add(Algo::ArStaged, 0, 256, 2);
      }
      if (nvls && n >= 2)
        for (const auto& sh : kNvlsShapes)
          if (sh[4] == 0 || n >= 4)  // copy-in first measured slower on 2 GPUs
            v.push_back({Algo::ArNvls, 0, 0, 0, 0, 0, 0, pack_nvls_shape(sh[0], sh[1], sh[2], sh[3], sh[4])});
      v.push_back({Algo::ArPush, 0, 0, 0, 0});
      break;
    case Kind::ReduceScatter:
      if (nvls && n >= 2) v.push_back({Algo::RsNvls, 0, 0, 0, 0});
      add(Algo::RsPull, 0);
      v.push_back({Algo::RsLL, 0, 0, 0, 0});
      v.push_back({Algo::RsPush, 0, 0, 0, 0});
      if (small) {
        add(Algo::RsStaged, 0, 64, 3);
        add(Algo::RsStaged, 0, 128, 2);
        add(Algo::RsStaged, 0, 256, 2);
      }
      break;
    case Kind::AllGather:
      if (nvls && n >= 2) v.push_back({Algo::AgNvls, 0, 0, 0, 0});
      add(Algo::AgPull, 0);
      add(Algo::AgPush, 0);
      v.push_back({Algo::AgLL, 0, 0, 0, 0});
      if (small) add(Algo::AgPull, 10000);
      break;
    case Kind::Broadcast:
      if (nvls && n >= 2) v.push_back({Algo::BcNvls, 0, 0, 0, 0});
      if (n >= 3) add(Algo::BcScatter, 0);
      if (small) {
        add(Algo::BcPull, 0);
        add(Algo::BcPull, 10000);
      }
      v.push_back({Algo::BcRing, 0, 0, 0, 0});
      v.push_back({Algo::BcLL, 0, 0, 0, 0});
      if (n >= 3) {
        add(Algo::BcChain, 10000, 64, 0);
        add(Algo::BcChain, 10000, 128, 0);
        add(Algo::BcChain, 0, 128, 0);
      }
      break;
    default:
      break;
  }
  return v;
}

double busbw_factor(Kind k, int n) {
  if (n <= 1) return 1.0;
  if (k == Kind::AllReduce) return 2.0 * (n - 1) / n;
  if (k == Kind::AllGather || k == Kind::ReduceScatter) return double(n - 1) / n;
  return 1.0;
}

}  // namespace

void tune_routes(const int* devices, int n, size_t bytes, CalibResult* out) {
  Runtime& r = rt();
  if (n < 2) return;
  bytes = (bytes / (size_t(n) * 256)) * size_t(n) * 256;
  std::vector<void*> send(size_t(n), nullptr), recv(size_t(n), nullptr);
  std::vector<cudaStream_t> streams(size_t(n), nullptr);
  std::vector<cudaEvent_t> e0(size_t(n), nullptr), e1(size_t(n), nullptr);
  bool ok = true;
  for (int i = 0; i < n && ok; ++i) {
    ok = cudaSetDevice(devices[i]) == cudaSuccess && cudaMalloc(&send[size_t(i)], bytes) == cudaSuccess &&
         cudaMalloc(&recv[size_t(i)], bytes) == cudaSuccess &&
         cudaMemset(send[size_t(i)], 0, bytes) == cudaSuccess &&
         cudaStreamCreateWithFlags(&streams[size_t(i)], cudaStreamNonBlocking) == cudaSuccess &&
         cudaEventCreate(&e0[size_t(i)]) == cudaSuccess && cudaEventCreate(&e1[size_t(i)]) == cudaSuccess;
  }
  const bool nvls = r.policy.nvls != NvlsMode::Off && nvls_supported(devices, n);
  // Two tuning sizes: the large one (the policy's) and a small one; the
  // small choice serves messages below their geometric mean.
  // A third, tiny size (1 MiB) picks among the SM routes for small messages,
  // where launch and synchronization latency outweigh the bytes.
  const size_t unit = size_t(n) * 256;
  const size_t small_bytes = std::max(unit, (size_t(64) << 20) / unit * unit);
  const size_t tiny_bytes = std::max(unit, (size_t(1) << 20) / unit * unit);
  const bool two_sizes = bytes >= 4 * small_bytes;
  for (int pass = 0; pass < (two_sizes ? 3 : 1); ++pass) {
    const size_t size = pass == 0 ? bytes : pass == 1 ? small_bytes : tiny_bytes;
    for (int kk = 0; ok && kk < int(Kind::Count); ++kk) {
      const Kind kind = Kind(kk);
      CliqueDesc d;
      d.kind = kind;
      d.dtype = DType::F32;
      d.op = RedOp::Sum;
      d.nranks = n;
      d.bytes = (kind == Kind::AllGather || kind == Kind::ReduceScatter) ? size / size_t(n) : size;
      d.count = d.bytes / 4;
      d.root = 0;
      Binding b;
      b.nranks = n;
      b.fold.dtype = DType::F32;
      b.fold.op = RedOp::Sum;
      b.fold.nranks = n;
      for (int i = 0; i < n; ++i) {
        b.device[i] = devices[i];
        b.stream[i] = streams[size_t(i)];
        b.send[i] = send[size_t(i)];
        b.recv[i] = recv[size_t(i)];
      }
      double best_ms = 1e30, best_real_ms = 1e30;
      Candidate best{Algo::Fallback, -1, -1, 0, 0};
      for (const Candidate& c : pass == 2 ? tiny_candidates(kind, n, nvls) : candidates(kind, n, nvls, *out)) {
        Shares s;
        s.ce_ppm = c.ce_ppm;
        s.host_ppm = c.host_ppm;
        s.stage_piece = size_t(c.piece_mib) << 20;
        s.stage_depth = c.depth;
        s.split_ppm = c.split_ppm;
        s.split_blocks = c.split_blocks;
        unpack_nvls_shape(c.nvls_shape, &s);
        Plan plan;
        build_plan(c.algo, d, r.policy, s, plan);
        std::string why;
        if (!r.exec.ensure(plan.needs, devices, n, &why)) {
          cudaGetLastError();
          continue;
        }
        bool good = true;
        float ms = 0;
        for (int rep = 0; rep < 2 && good; ++rep) {  // rep 0 warms up
          for (int i = 0; i < n; ++i) {
            cudaSetDevice(devices[i]);
            cudaEventRecord(e0[size_t(i)], streams[size_t(i)]);
          }
          const int runs = rep ? 3 : 1;
          for (int k = 0; k < runs && good; ++k) {
            cudaError_t err = cudaSuccess;
            good = r.exec.execute(plan, b, &err, nullptr) == ExecStatus::Ok;
          }
          float worst = 0;
          for (int i = 0; i < n && good; ++i) {
            cudaSetDevice(devices[i]);
            cudaEventRecord(e1[size_t(i)], streams[size_t(i)]);
          }
          for (int i = 0; i < n && good; ++i) {
            cudaSetDevice(devices[i]);
            float t = 0;
            good = cudaEventSynchronize(e1[size_t(i)]) == cudaSuccess &&
                   cudaEventElapsedTime(&t, e0[size_t(i)], e1[size_t(i)]) == cudaSuccess;
            worst = t > worst ? t : worst;
          }
          ms = worst / float(runs);
        }
        if (!good) {
          cudaGetLastError();
          r.exec.drain(devices, n);
          continue;
        }
        char line[240];
        const size_t logical = (kind == Kind::AllGather || kind == Kind::ReduceScatter) ? size : d.bytes;
        std::snprintf(line, sizeof line,
                      "tune %s n=%d bytes=%zu %s ce_ppm=%d host_ppm=%d piece_mib=%d depth=%d split=%d/%d "
                      "nvls_shape=%d busbw_gbs=%.1f",
                      kind_name(kind), n, logical, algo_name(c.algo), c.ce_ppm, c.host_ppm, c.piece_mib,
                      c.depth, c.split_ppm, c.split_blocks, c.nvls_shape,
                      logical / (ms * 1e-3) / 1e9 * busbw_factor(kind, n));
        r.summary.note(line);
        // An event-ordered chain pays a cross-GPU event wait per piece and hop,
        // so its rate drops as messages outgrow the tuning size (measured at 4
        // ranks: equal to the in-kernel push chain at 4 GiB, 10 % behind at
        // 8 GiB); it must win by 3 % to be chosen.
        const float score = c.algo == Algo::BcChain ? ms * 1.03f : ms;
        if (score < best_ms) {
          best_ms = score;
          best_real_ms = ms;
          best = c;
        }
      }
      if (best.algo != Algo::Fallback && pass == 2) {
        out->tiny_pref[kk] = int(best.algo);
      } else if (best.algo != Algo::Fallback && pass == 1) {
        out->small_pref[kk] = int(best.algo);
        out->small_ce_ppm[kk] = best.ce_ppm;
        out->small_host_ppm[kk] = best.host_ppm;
        out->small_piece_mib[kk] = best.piece_mib;
        out->small_depth[kk] = best.depth;
        out->small_split_ppm[kk] = best.split_ppm;
        out->small_split_blocks[kk] = best.split_blocks;
        out->small_nvls_shape[kk] = best.nvls_shape;
      } else if (best.algo != Algo::Fallback) {
        out->preferred[kk] = int(best.algo);
        out->ce_ppm[kk] = best.ce_ppm;
        out->host_ppm[kk] = best.host_ppm;
        out->stage_piece_mib[kk] = best.piece_mib;
        out->stage_depth[kk] = best.depth;
        out->split_ppm[kk] = best.split_ppm;
        out->split_blocks[kk] = best.split_blocks;
        out->nvls_shape[kk] = best.nvls_shape;
        const size_t logical = (kind == Kind::AllGather || kind == Kind::ReduceScatter) ? size : d.bytes;
        out->route_gbs[kk] = logical / (best_real_ms * 1e-3) / 1e9 * busbw_factor(kind, n);
      }
    }
  }
  if (two_sizes) {
    const double mean = std::sqrt(double(small_bytes) * double(bytes));
    out->small_below_mib = int(mean / double(1 << 20));
    out->tiny_below_kib = int(std::sqrt(double(tiny_bytes) * double(small_bytes)) / 1024.0);
  }
  for (int i = 0; i < n; ++i) {
    cudaSetDevice(devices[i]);
    cudaDeviceSynchronize();
    if (send[size_t(i)]) cudaFree(send[size_t(i)]);
    if (recv[size_t(i)]) cudaFree(recv[size_t(i)]);
    if (streams[size_t(i)]) cudaStreamDestroy(streams[size_t(i)]);
    if (e0[size_t(i)]) cudaEventDestroy(e0[size_t(i)]);
    if (e1[size_t(i)]) cudaEventDestroy(e1[size_t(i)]);
  }
  cudaGetLastError();
}

void tune_single(int device, size_t bytes, CalibResult* out) {
  Runtime& r = rt();
  bytes = bytes / 256 * 256;
  if (!bytes) return;
  void* send = nullptr;
  void* recv = nullptr;
  cudaStream_t stream = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  bool ok = cudaSetDevice(device) == cudaSuccess && cudaMalloc(&send, bytes) == cudaSuccess &&
            cudaMalloc(&recv, bytes) == cudaSuccess && cudaMemset(send, 0, bytes) == cudaSuccess &&
            cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) == cudaSuccess &&
            cudaEventCreate(&e0) == cudaSuccess && cudaEventCreate(&e1) == cudaSuccess;
  const int devices[1] = {device};
  CliqueDesc d;
  d.kind = Kind::AllReduce;
  d.dtype = DType::F32;
  d.op = RedOp::Sum;
  d.nranks = 1;
  d.bytes = bytes;
  d.count = bytes / 4;
  Binding b;
  b.nranks = 1;
  b.device[0] = device;
  b.stream[0] = stream;
  b.send[0] = send;
  b.recv[0] = recv;
  b.fold.dtype = DType::F32;
  b.fold.nranks = 1;
  double best_ms = 1e30;
  int best_ce = -1;
  // The kernel alone, and beside copy-engine shares of the leading bytes.
  for (int ce : {0, 1500, 2500, 3500}) {
    if (!ok) break;
    Shares s;
    s.ce_ppm = ce;
    Plan plan;
    build_plan(Algo::ArTwoShot, d, r.policy, s, plan);
    std::string why;
    if (!r.exec.ensure(plan.needs, devices, 1, &why)) {
      cudaGetLastError();
      continue;
    }
    bool good = true;
    float ms = 0;
    for (int rep = 0; rep < 2 && good; ++rep) {  // rep 0 warms up
      const int runs = rep ? 5 : 2;
      good = cudaEventRecord(e0, stream) == cudaSuccess;
      for (int k = 0; k < runs && good; ++k) {
        cudaError_t err = cudaSuccess;
        good = r.exec.execute(plan, b, &err, nullptr) == ExecStatus::Ok;
      }
      good = good && cudaEventRecord(e1, stream) == cudaSuccess && cudaEventSynchronize(e1) == cudaSuccess &&
             cudaEventElapsedTime(&ms, e0, e1) == cudaSuccess;
      ms /= float(runs);
    }
    if (!good) {
      cudaGetLastError();
      r.exec.drain(devices, 1);
      continue;
    }
    char line[128];
    std::snprintf(line, sizeof line, "tune local-copy n=1 bytes=%zu ce_ppm=%d algbw_gbs=%.1f", bytes, ce,
                  bytes / (ms * 1e-3) / 1e9);
    r.summary.note(line);
    if (ms < best_ms) {
      best_ms = ms;
      best_ce = ce;
    }
  }
  if (best_ce >= 0) {
    out->valid = true;
    for (int k = 0; k < 4; ++k) {
      out->preferred[k] = int(Algo::ArTwoShot);  // unused at one rank (every kind is the copy)
      out->ce_ppm[k] = best_ce;
      out->host_ppm[k] = 0;
      out->route_gbs[k] = bytes / (best_ms * 1e-3) / 1e9;
    }
  }
  cudaSetDevice(device);
  cudaDeviceSynchronize();
  if (send) cudaFree(send);
  if (recv) cudaFree(recv);
  if (stream) cudaStreamDestroy(stream);
  if (e0) cudaEventDestroy(e0);
  if (e1) cudaEventDestroy(e1);
  cudaGetLastError();
}

}  // namespace nb
