#include "core/calib_model.h"

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace nb {

bool small_message(const CalibResult& c, size_t logical) {
  return c.small_below_mib > 0 && logical < (size_t(c.small_below_mib) << 20);
}

bool tiny_message(const CalibResult& c, size_t logical) {
  return c.tiny_below_kib > 0 && logical < (size_t(c.tiny_below_kib) << 10);
}

Algo tuned_route(const CalibResult& c, int kind, size_t logical) {
  if (kind < 0 || kind >= 4) return Algo::Fallback;
  if (tiny_message(c, logical) && c.tiny_pref[kind] != 0) return Algo(c.tiny_pref[kind]);
  if (small_message(c, logical) && c.small_pref[kind] != 0) return Algo(c.small_pref[kind]);
  return Algo(c.preferred[kind]);
}

Shares shares_from(const CalibResult& c, Algo a, int n, bool small) {
  Shares s;
  if (!c.valid || n < 2 || c.nvlink_sm_gbs <= 0) return s;
  const double N = double(n);
  const double bnv = c.nvlink_sm_gbs;
  const double bp = std::min(c.pcie_d2h_gbs, c.pcie_h2d_gbs);
  const double bf = c.fold_gbs;
  // NVLink seconds per byte of this GPU's share, and host seconds per byte.
  double nv = 0, host = 0;
  switch (a) {
    case Algo::ArTwoShot:
      nv = 2.0 * (N - 1.0) / N / bnv;
      host = std::max(bp > 0 ? 1.0 / bp : 1e30, bf > 0 ? N / bf : 1e30);
      break;
    case Algo::RsPull:
      nv = (N - 1.0) / bnv;
      host = std::max(bp > 0 ? N / bp : 1e30, bf > 0 ? N * N / bf : 1e30);
      break;
    case Algo::AgPull:
      nv = (N - 1.0) / bnv;
      host = bp > 0 ? (N - 1.0) / bp : 1e30;
      break;
    case Algo::BcPull: case Algo::BcScatter:
      nv = 1.0 / bnv;
      host = bp > 0 ? 1.0 / bp : 1e30;
      break;
    default:
      return s;
  }
  double h = nv / (nv + host);
  if (h < 0.03) h = 0;  // the predicted gain is about h: not worth the lanes
  h = std::min(h, 0.25);
  s.host_ppm = int(h * 10000.0);
  const bool ce_algo = a == Algo::ArTwoShot || a == Algo::AgPull || a == Algo::BcPull ||
                       a == Algo::BcScatter;
  if (ce_algo && c.nvlink_mix_gbs > 1.03 * bnv && c.mix_ce_fraction > 0)
    s.ce_ppm = int(std::min(0.5, c.mix_ce_fraction) * 10000.0);
  // A measured route choice overrides the model for that route (the
  // small-size choice for a small message, when it is this route).
  for (int k = 0; k < 4; ++k) {
    if (small && c.small_pref[k] == int(a)) {
      if (c.small_ce_ppm[k] >= 0) s.ce_ppm = c.small_ce_ppm[k];
      if (c.small_host_ppm[k] >= 0) s.host_ppm = c.small_host_ppm[k];
      if (c.small_piece_mib[k] > 0) s.stage_piece = size_t(c.small_piece_mib[k]) << 20;
      if (c.small_depth[k] > 0) s.stage_depth = c.small_depth[k];
      if (c.small_split_ppm[k] > 0) s.split_ppm = c.small_split_ppm[k];
      if (c.small_split_blocks[k] > 0) s.split_blocks = c.small_split_blocks[k];
      if (c.small_nvls_shape[k] > 0) unpack_nvls_shape(c.small_nvls_shape[k], &s);
      continue;
    }
    if (c.preferred[k] != int(a)) continue;
    if (c.ce_ppm[k] >= 0) s.ce_ppm = c.ce_ppm[k];
    if (c.host_ppm[k] >= 0) s.host_ppm = c.host_ppm[k];
    if (c.stage_piece_mib[k] > 0) s.stage_piece = size_t(c.stage_piece_mib[k]) << 20;
    if (c.stage_depth[k] > 0) s.stage_depth = c.stage_depth[k];
    if (c.split_ppm[k] > 0) s.split_ppm = c.split_ppm[k];
    if (c.split_blocks[k] > 0) s.split_blocks = c.split_blocks[k];
    if (c.nvls_shape[k] > 0) unpack_nvls_shape(c.nvls_shape[k], &s);
  }
  return s;
}

std::string calib_to_json(const CalibResult& c, const std::string& key) {
  char buf[1536];
  std::snprintf(buf, sizeof buf,
                "{\"key\": \"%s\", \"nvlink_sm_gbs\": %.3f, \"nvlink_ce_gbs\": %.3f, "
                "\"nvlink_mix_gbs\": %.3f, \"mix_ce_fraction\": %.5f, \"pcie_d2h_gbs\": %.3f, "
                "\"pcie_h2d_gbs\": %.3f, \"fold_gbs\": %.3f",
                key.c_str(), c.nvlink_sm_gbs, c.nvlink_ce_gbs, c.nvlink_mix_gbs, c.mix_ce_fraction,
                c.pcie_d2h_gbs, c.pcie_h2d_gbs, c.fold_gbs);
  std::string s = buf;
  for (int k = 0; k < 4; ++k) {
    std::snprintf(buf, sizeof buf,
                  ", \"pref%d\": %d, \"ce%d\": %d, \"host%d\": %d, \"piece%d\": %d, \"depth%d\": %d",
                  k, c.preferred[k], k, c.ce_ppm[k], k, c.host_ppm[k], k, c.stage_piece_mib[k], k,
                  c.stage_depth[k]);
    s += buf;
    std::snprintf(buf, sizeof buf,
                  ", \"spref%d\": %d, \"sce%d\": %d, \"shost%d\": %d, \"spiece%d\": %d, \"sdepth%d\": %d",
                  k, c.small_pref[k], k, c.small_ce_ppm[k], k, c.small_host_ppm[k], k,
                  c.small_piece_mib[k], k, c.small_depth[k]);
    s += buf;
  }
  std::snprintf(buf, sizeof buf, ", \"small_below_mib\": %d, \"tiny_below_kib\": %d", c.small_below_mib,
                c.tiny_below_kib);
  s += buf;
  for (int k = 0; k < 4; ++k) {
    std::snprintf(buf, sizeof buf,
                  ", \"tpref%d\": %d, \"split%d\": %d, \"sblocks%d\": %d, \"ssplit%d\": %d, "
                  "\"ssblocks%d\": %d, \"engage%d\": %d, \"nvshape%d\": %d, \"snvshape%d\": %d",
                  k, c.tiny_pref[k], k, c.split_ppm[k], k, c.split_blocks[k], k, c.small_split_ppm[k], k,
                  c.small_split_blocks[k], k, c.engage_kib[k], k, c.nvls_shape[k], k, c.small_nvls_shape[k]);
    s += buf;
  }
  return s + "}\n";
}

static bool json_number(const std::string& text, const char* name, double* out) {
  const std::string pat = std::string("\"") + name + "\":";
  const size_t p = text.find(pat);
  if (p == std::string::npos) return false;
  const char* s = text.c_str() + p + pat.size();
  char* end = nullptr;
  const double v = std::strtod(s, &end);
  if (end == s) return false;
  *out = v;
  return true;
}

bool calib_from_json(const std::string& text, const std::string& key, CalibResult* out) {
  const std::string pat = "\"key\": \"" + key + "\"";
  if (text.find(pat) == std::string::npos) return false;
  CalibResult c;
  bool ok = json_number(text, "nvlink_sm_gbs", &c.nvlink_sm_gbs) &&
            json_number(text, "nvlink_ce_gbs", &c.nvlink_ce_gbs) &&
            json_number(text, "nvlink_mix_gbs", &c.nvlink_mix_gbs) &&
            json_number(text, "mix_ce_fraction", &c.mix_ce_fraction) &&
            json_number(text, "pcie_d2h_gbs", &c.pcie_d2h_gbs) &&
            json_number(text, "pcie_h2d_gbs", &c.pcie_h2d_gbs) &&
            json_number(text, "fold_gbs", &c.fold_gbs);
  if (!ok) return false;
  for (int k = 0; k < 4; ++k) {
    double v = 0;
    const std::string K = std::to_string(k);
    if (json_number(text, ("pref" + K).c_str(), &v)) c.preferred[k] = int(v);
    if (json_number(text, ("ce" + K).c_str(), &v)) c.ce_ppm[k] = int(v);
    if (json_number(text, ("host" + K).c_str(), &v)) c.host_ppm[k] = int(v);
    if (json_number(text, ("piece" + K).c_str(), &v)) c.stage_piece_mib[k] = int(v);
    if (json_number(text, ("depth" + K).c_str(), &v)) c.stage_depth[k] = int(v);
    if (json_number(text, ("spref" + K).c_str(), &v)) c.small_pref[k] = int(v);
    if (json_number(text, ("sce" + K).c_str(), &v)) c.small_ce_ppm[k] = int(v);
    if (json_number(text, ("shost" + K).c_str(), &v)) c.small_host_ppm[k] = int(v);
    if (json_number(text, ("spiece" + K).c_str(), &v)) c.small_piece_mib[k] = int(v);
    if (json_number(text, ("sdepth" + K).c_str(), &v)) c.small_depth[k] = int(v);
  }
  {
    double v = 0;
    if (json_number(text, "small_below_mib", &v)) c.small_below_mib = int(v);
    if (json_number(text, "tiny_below_kib", &v)) c.tiny_below_kib = int(v);
    for (int k = 0; k < 4; ++k) {
      const std::string K = std::to_string(k);
      if (json_number(text, ("tpref" + K).c_str(), &v)) c.tiny_pref[k] = int(v);
      if (json_number(text, ("split" + K).c_str(), &v)) c.split_ppm[k] = int(v);
      if (json_number(text, ("sblocks" + K).c_str(), &v)) c.split_blocks[k] = int(v);
      if (json_number(text, ("ssplit" + K).c_str(), &v)) c.small_split_ppm[k] = int(v);
      if (json_number(text, ("ssblocks" + K).c_str(), &v)) c.small_split_blocks[k] = int(v);
      if (json_number(text, ("engage" + K).c_str(), &v)) c.engage_kib[k] = int(v);
      if (json_number(text, ("nvshape" + K).c_str(), &v)) c.nvls_shape[k] = int(v);
      if (json_number(text, ("snvshape" + K).c_str(), &v)) c.small_nvls_shape[k] = int(v);
    }
  }
  c.valid = true;
  *out = c;
  return true;
}

}  // namespace nb
