// Pure part of path calibration: the measured rates, the share model that
// turns them into per-algorithm byte splits, and the JSON cache format.
//
// Share model. For each algorithm, per GPU, the SM/NVLink part carries
// c_nv bytes of NVLink traffic per byte of its share at B_nv, the host part
// carries c_h bytes of PCIe traffic per byte at B_pcie (plus, for reductions,
// N bytes of host-fold input per byte at B_fold, over all GPUs at once); the
// host share h balances the two times, and is dropped when the predicted gain
// is under 3 %. The copy-engine share is the CE part of the measured mixed
// SM+CE rate, used only when the mix beats SM pulls alone by 3 % or more.
//
// Parity: replaces the reference's constant divisors 7/7/7/7/6 and piece
// sizes (shim/nccl_collectives_shim.cu:51-91).
#pragma once

#include <string>

#include "core/plan.h"

namespace nb {

struct CalibResult {
  bool valid = false;
  double nvlink_sm_gbs = 0;   // per-GPU inbound, SM pulls, all GPUs pulling
  double nvlink_ce_gbs = 0;   // per-GPU inbound, copy engine alone
  double nvlink_mix_gbs = 0;  // per-GPU inbound, SM + CE together
  double mix_ce_fraction = 0; // CE's part of the mixed rate
  double pcie_d2h_gbs = 0;    // per GPU, every GPU at once, D2H and H2D together
  double pcie_h2d_gbs = 0;
  double fold_gbs = 0;        // host fold input throughput (all threads)
  // Route tuning: the fastest measured algorithm per collective kind and
  // its copy-engine share (parts per 10000), -1 / Fallback when untuned.
  int preferred[4] = {0, 0, 0, 0};
  int ce_ppm[4] = {-1, -1, -1, -1};
  int host_ppm[4] = {-1, -1, -1, -1};
  int stage_piece_mib[4] = {0, 0, 0, 0};
  int stage_depth[4] = {0, 0, 0, 0};
  double route_gbs[4] = {0, 0, 0, 0};  // busbw of the chosen route at the tuning size
  int split_ppm[4] = {0, 0, 0, 0};     // hybrid routes: the switch's share and blocks
  int split_blocks[4] = {0, 0, 0, 0};
  int nvls_shape[4] = {0, 0, 0, 0};    // NVLS routes: packed kernel shape (see pack_nvls_shape)
  // The same, tuned at a small size: used for messages below small_below_mib
  // (0 = no small-size choice). Pipelined routes pay a start-up that only
  // large messages amortize, so the best route differs with size.
  int small_pref[4] = {0, 0, 0, 0};
  int small_ce_ppm[4] = {-1, -1, -1, -1};
  int small_host_ppm[4] = {-1, -1, -1, -1};
  int small_piece_mib[4] = {0, 0, 0, 0};
  int small_depth[4] = {0, 0, 0, 0};
  int small_split_ppm[4] = {0, 0, 0, 0};
  int small_split_blocks[4] = {0, 0, 0, 0};
  int small_nvls_shape[4] = {0, 0, 0, 0};
  int small_below_mib = 0;
  // A third band for small messages, tuned among the SM routes only (no
  // pipelines, no copy-engine or host shares): used below tiny_below_kib.
  int tiny_pref[4] = {0, 0, 0, 0};
  int tiny_below_kib = 0;
  // Measured crossover with NCCL (after the communicators exist): the
  // smallest logical size, in KiB, from which the tuned routes were faster
  // at every size of the ladder up to the policy threshold (0 = not measured).
  int engage_kib[4] = {0, 0, 0, 0};
};

// An NVLS kernel shape in one int: (ramp + 3 * ahead) * 2 * 10^8 + movers
// (threads, below 2000) * 10^5 + unroll * 10^4 + round MiB. Each part 0 =
// the policy's; ramp 1 = uniform AllReduce rounds, 2 = ramped first and
// last rounds; ahead 1 = the copier's usual order, 2 = every copy-in first.
inline int pack_nvls_shape(int movers, int unroll, int round_mib, int ramp = 0, int ahead = 0) {
  return (ramp + 3 * ahead) * 200000000 + movers * 100000 + unroll * 10000 + round_mib;
}
inline void unpack_nvls_shape(int v, Shares* s) {
  const int sched = v / 200000000;
  s->nvls_ramp = sched % 3;
  s->nvls_ahead = sched / 3;
  v %= 200000000;
  s->nvls_movers = v / 100000;
  s->nvls_unroll = (v / 10000) % 10;
  s->nvls_round_mib = v % 10000;
}

// Whether a message of `logical` bytes takes the small-size choice.
bool small_message(const CalibResult& c, size_t logical);
// Whether it takes the tiny-size choice (a route of the small band's own).
bool tiny_message(const CalibResult& c, size_t logical);
// The tuned route of `kind` for a message of `logical` bytes (Fallback when
// untuned).
Algo tuned_route(const CalibResult& c, int kind, size_t logical);
// Byte shares of route `a`; `small` selects the small-size tuning's shares.
Shares shares_from(const CalibResult& c, Algo a, int n, bool small = false);
std::string calib_to_json(const CalibResult& c, const std::string& key);
bool calib_from_json(const std::string& text, const std::string& key, CalibResult* out);

}  // namespace nb
