#include "core/plan.h"

#include <algorithm>

namespace nb {

bool operator==(StreamId a, StreamId b) {
  return a.kind == b.kind && a.dev == b.dev && a.lane == b.lane;
}
bool operator==(EventId a, EventId b) {
  return a.kind == b.kind && a.dev == b.dev && a.lane == b.lane && a.index == b.index;
}

void Needs::merge(const Needs& o) {
  lanes = std::max(lanes, o.lanes);
  bounce_bytes = std::max(bounce_bytes, o.bounce_bytes);
  phase_events = std::max(phase_events, o.phase_events);
  nvls_bytes = std::max(nvls_bytes, o.nvls_bytes);
  temp_bytes = std::max(temp_bytes, o.temp_bytes);
  ring = ring || o.ring;
  pushred = pushred || o.pushred;
  oneshot = oneshot || o.oneshot;
}

void slice_of(size_t bytes, int parts, int i, size_t* off, size_t* len) {
  const size_t base = (bytes / size_t(parts)) & ~size_t(31);
  *off = base * size_t(i);
  *len = i == parts - 1 ? bytes - *off : base;
}

size_t host_share(size_t len, int ppm, const Policy& p) {
  if (ppm <= 0 || len == 0) return 0;
  const size_t h = (size_t((unsigned __int128)len * unsigned(ppm) / 10000) / 16) * 16;
  return h >= p.min_host_bytes ? h : 0;
}

size_t ce_share(size_t len, int ppm) {
  if (ppm <= 0 || len == 0) return 0;
  return (size_t((unsigned __int128)len * unsigned(ppm) / 10000) / 16) * 16;
}

namespace {

StreamId caller(int r) { return {Strm::Caller, uint8_t(r), 0}; }
StreamId d2h(int r, int lane) { return {Strm::D2H, uint8_t(r), uint8_t(lane)}; }
StreamId h2d(int r, int lane) { return {Strm::H2D, uint8_t(r), uint8_t(lane)}; }
StreamId host(int lane) { return {Strm::Host, 0, uint8_t(lane)}; }
EventId input_ready(int r) { return {Ev::InputReady, uint8_t(r), 0, 0}; }
EventId join_done(int r) { return {Ev::Join, uint8_t(r), 0, 0}; }
EventId done(StreamId s) { return {Ev::Done, s.dev, s.lane, uint16_t(s.kind)}; }
EventId d2h_done(int r, int lane) { return {Ev::D2HDone, uint8_t(r), uint8_t(lane), 0}; }
EventId h2d_done(int r, int lane) { return {Ev::H2DDone, uint8_t(r), uint8_t(lane), 0}; }
EventId host_done(int lane) { return {Ev::HostDone, 0, uint8_t(lane), 0}; }
EventId lane_free(int lane) { return {Ev::LaneFree, 0, uint8_t(lane), 0}; }

// Appends ops and tracks, per stream, which ranks' InputReady it has already
// waited for, and which internal streams each rank used (for the join).
class Builder {
 public:
  Builder(Plan& plan, Algo algo, const CliqueDesc& d, const Policy& p) : p_(plan), pol_(p) {
    p_.algo = algo;
    p_.desc = d;
    p_.ops.clear();
    p_.needs = Needs{};
    p_.sm_bytes = p_.ce_bytes = p_.host_bytes = 0;
    n_ = d.nranks;
  }
  int n() const { return n_; }
  const Policy& policy() const { return pol_; }
  Plan& plan() { return p_; }

  void record(EventId e, StreamId s) {
    if (e.kind == Ev::Phase) p_.needs.phase_events = std::max<uint16_t>(p_.needs.phase_events, uint16_t(e.index + 1));
    PlanOp op;
    op.kind = OpKind::Record;
    op.stream = s;
    op.event = e;
    p_.ops.push_back(op);
  }
  void wait(StreamId s, EventId e) {
    PlanOp op;
    op.kind = OpKind::Wait;
    op.stream = s;
    op.event = e;
    p_.ops.push_back(op);
  }
  // `s` is about to touch rank r's buffers: make it wait r's InputReady once
  // (with a hub: the hub's AllReady, once per stream).
  void touch(StreamId s, int r) {
    if (s.kind == Strm::Caller && s.dev == r) return;  // stream order
    if (hub_) {
      for (const auto& t : hub_waiters_)
        if (t == s) return;
      hub_waiters_.push_back(s);
      wait(s, {Ev::AllReady, 0, 0, 0});
      use(s);
      return;
    }
    for (const auto& t : touched_)
      if (t.first == s && t.second == r) return;
    touched_.push_back({s, r});
    wait(s, input_ready(r));
    use(s);
  }
  void use(StreamId s) {
    if (s.kind == Strm::Caller || s.kind == Strm::Host || s.kind == Strm::Hub) return;
    for (const auto& u : used_)
      if (u == s) return;
    used_.push_back(s);
  }
  void ce_copy(StreamId s, Loc dst, Loc src, size_t bytes) {
    if (!bytes) return;
    PlanOp op;
    op.kind = OpKind::CeCopy;
    op.stream = s;
    op.nsrc = op.ndst = 1;
    op.src[0] = src;
    op.dst[0] = dst;
    op.len[0] = op.bytes = bytes;
    p_.ops.push_back(op);
    use(s);
  }
  void sm_copy(StreamId s, const Loc* dst, const Loc* src, const size_t* len, int nseg) {
    PlanOp op;
    op.kind = OpKind::SmCopy;
    op.stream = s;
    for (int i = 0; i < nseg; ++i) {
      if (!len[i]) continue;
      op.src[op.nsrc] = src[i];
      op.dst[op.ndst] = dst[i];
      op.len[op.nsrc] = len[i];
      op.bytes += len[i];
      ++op.nsrc;
      ++op.ndst;
    }
    if (!op.nsrc) return;
    p_.ops.push_back(op);
    use(s);
  }
  void sm_reduce(StreamId s, const Loc* src, int nsrc, const Loc* dst, int ndst, size_t bytes) {
    if (!bytes) return;
    PlanOp op;
    op.kind = OpKind::SmReduce;
    op.stream = s;
    op.nsrc = uint8_t(nsrc);
    op.ndst = uint8_t(ndst);
    for (int i = 0; i < nsrc; ++i) op.src[i] = src[i];
    for (int i = 0; i < ndst; ++i) op.dst[i] = dst[i];
    op.len[0] = op.bytes = bytes;
    p_.ops.push_back(op);
    use(s);
  }
  void host_reduce(StreamId s, const Loc* src, int nsrc, Loc dst, size_t bytes) {
    PlanOp op;
    op.kind = OpKind::HostReduce;
    op.stream = s;
    op.nsrc = uint8_t(nsrc);
    op.ndst = 1;
    for (int i = 0; i < nsrc; ++i) op.src[i] = src[i];
    op.dst[0] = dst;
    op.len[0] = op.bytes = bytes;
    p_.ops.push_back(op);
  }
  void nvls(StreamId s, int r, size_t bytes, size_t off = 0, uint16_t grid = 0) {
    PlanOp op;
    op.kind = OpKind::NvlsReduce;
    op.stream = s;
    op.nsrc = op.ndst = 1;
    op.src[0] = send_at(r, off);
    op.dst[0] = recv_at(r, off);
    op.len[0] = op.bytes = bytes;
    op.grid = grid;
    p_.ops.push_back(op);
    use(s);
  }

  // Every rank records InputReady. From four ranks on, a hub stream on rank
  // 0's GPU waits for all of them and records AllReady, so a stream that
  // touches peers waits on one event instead of N - 1: the cross-device
  // event fans cost O(N) host calls instead of O(N^2).
  void prologue() {
    for (int r = 0; r < n_; ++r) record(input_ready(r), caller(r));
    if (n_ >= kHubRanks) {
      hub_ = true;
      const StreamId h{Strm::Hub, 0, 0};
      for (int r = 0; r < n_; ++r) wait(h, input_ready(r));
      record({Ev::AllReady, 0, 0, 0}, h);
    }
  }
  // Gang engines launched on caller streams share state across calls (see
  // Ev::GangDone): every rank's caller stream first waits for the previous
  // gang call to have finished on every GPU of the clique.
  void gang_fence() {
    for (int r = 0; r < n_; ++r)
      for (int q = 0; q < n_; ++q) wait(caller(r), {Ev::GangDone, uint8_t(q), 0, 0});
  }
  void gang_done(int r) { record({Ev::GangDone, uint8_t(r), 0, 0}, caller(r)); }
  // Every rank's caller stream waits for its own internal streams, then for
  // every peer's join, so no rank returns while a peer still reads its send
  // buffer or writes its receive buffer.
  void join() {
    for (int r = 0; r < n_; ++r) {
      for (const StreamId& s : used_) {
        if (s.dev != r) continue;
        record(done(s), s);
        wait(caller(r), done(s));
      }
      record(join_done(r), caller(r));
    }
    if (hub_) {
      const StreamId h{Strm::Hub, 0, 0};
      for (int r = 0; r < n_; ++r) wait(h, join_done(r));
      record({Ev::AllJoined, 0, 0, 0}, h);
      for (int r = 0; r < n_; ++r) wait(caller(r), {Ev::AllJoined, 0, 0, 0});
      return;
    }
    for (int r = 0; r < n_; ++r)
      for (int q = 0; q < n_; ++q)
        if (q != r) wait(caller(r), join_done(q));
  }

  // Stage `bytes` through the pinned-host lanes in pieces, round-robin over
  // lanes. For each piece: every source rank's D2H lands in its bounce
  // buffer; with `reduce` the host folds them (rank order) into HostOut;
  // every destination rank's H2D then copies the result (or, without
  // `reduce`, the single source's bounce) into its buffer. A lane is reused
  // only after all H2Ds of its previous piece completed (LaneFree), which is
  // the HostLaneReuse invariant.
  // srcs[i] / dsts[j] locate offset 0 of this staged range.
  void host_stage(const int* src_ranks, const Loc* srcs, int nsrc, const int* dst_ranks,
                  const Loc* dsts, int ndst, size_t bytes, bool reduce) {
    const size_t piece = pol_.host_piece;
    const int lanes = pol_.lanes;
    for (size_t rel = 0; rel < bytes; rel += piece) {
      const size_t cb = std::min(piece, bytes - rel);
      const int lane = int(pieces_++ % size_t(lanes));
      p_.needs.lanes = std::max(p_.needs.lanes, lane + 1);
      p_.needs.bounce_bytes = std::max(p_.needs.bounce_bytes, cb);
      Loc bounce[kMaxRanks];
      for (int i = 0; i < nsrc; ++i) {
        const int q = src_ranks[i];
        const StreamId s = d2h(q, lane);
        touch(s, q);
        wait(s, lane_free(lane));
        bounce[i] = bounce_at(q, lane);
        ce_copy(s, bounce[i], at(srcs[i], rel), cb);
        record(d2h_done(q, lane), s);
      }
      Loc out = bounce[0];
      if (reduce) {
        for (int i = 0; i < nsrc; ++i) wait(host(lane), d2h_done(src_ranks[i], lane));
        out = hostout_at(lane);
        host_reduce(host(lane), bounce, nsrc, out, cb);
        record(host_done(lane), host(lane));
      }
      for (int j = 0; j < ndst; ++j) {
        const int r = dst_ranks[j];
        const StreamId s = h2d(r, lane);
        touch(s, r);
        wait(s, reduce ? host_done(lane) : d2h_done(src_ranks[0], lane));
        ce_copy(s, at(dsts[j], rel), out, cb);
        record(h2d_done(r, lane), s);
      }
      for (int j = 0; j < ndst; ++j) wait(host(lane), h2d_done(dst_ranks[j], lane));
      if (!reduce)
        for (int i = 0; i < nsrc; ++i) wait(host(lane), d2h_done(src_ranks[i], lane));
      record(lane_free(lane), host(lane));
      p_.host_bytes += cb * size_t(nsrc + ndst);
    }
  }

 private:
  Plan& p_;
  const Policy& pol_;
  int n_ = 0;
  size_t pieces_ = 0;
  std::vector<std::pair<StreamId, int>> touched_;
  std::vector<StreamId> used_;
  bool hub_ = false;
  std::vector<StreamId> hub_waiters_;
  static constexpr int kHubRanks = 4;
};

void all_ranks(int n, int* ranks) {
  for (int i = 0; i < n; ++i) ranks[i] = i;
}

// AllReduce two-shot: rank r owns slice r. Its kernel reads slice r of every
// rank's input (fixed rank order), reduces in fp32 (fp64 for doubles) and
// stores the result into slice r of every rank's output: the reduce-scatter
// and all-gather halves of the ring, fused into one pass with no scratch.
// Optional copy-engine share: a middle part of each slice is reduced into the
// owner's output only, then pushed to the peers by the owner's copy engine.
// Optional host share: the slice's suffix goes through the host lanes.
// Over [base, base + total) of the buffers (the whole message by default;
// the hybrid route runs it on the part the switch does not take). `wrap`
// emits the prologue and the join.
void plan_ar_twoshot(Builder& b, const CliqueDesc& d, const Shares& s, size_t base = 0,
                     size_t total = ~size_t(0), bool wrap = true) {
  const int n = b.n();
  if (total == ~size_t(0)) total = d.bytes;
  if (wrap) b.prologue();
  int ranks[kMaxRanks];
  all_ranks(n, ranks);
  size_t off[kMaxRanks], len[kMaxRanks], host[kMaxRanks], ce[kMaxRanks];
  for (int r = 0; r < n; ++r) {
    slice_of(total, n, r, &off[r], &len[r]);
    off[r] += base;
    host[r] = n > 1 ? host_share(len[r], s.host_ppm, b.policy()) : 0;
    ce[r] = n > 1 ? ce_share(len[r] - host[r], s.ce_ppm) : 0;
  }
  for (int r = 0; r < n; ++r) {
    // Slice layout [copy-engine part | host part | SM part]: the first two
    // are whole 16-byte units, so every part starts 16-byte aligned and only
    // the SM part (last) can end in a partial vector.
    const size_t sm = len[r] - host[r] - ce[r];
    for (int q = 0; q < n; ++q) b.touch({Strm::Caller, uint8_t(r), 0}, q);
    if (ce[r]) {
      // Reduce the copy-engine part into this rank's output only, in
      // pieces, and push each piece to every peer from this GPU.
      const size_t piece = b.policy().sm_chunk;
      int k = 0;
      for (size_t rel = 0; rel < ce[r]; rel += piece, ++k) {
        const size_t cb = std::min(piece, ce[r] - rel);
        Loc src2[kMaxRanks];
        for (int q = 0; q < n; ++q) src2[q] = send_at(q, off[r] + rel);
        Loc own = recv_at(r, off[r] + rel);
        b.sm_reduce({Strm::Caller, uint8_t(r), 0}, src2, n, &own, 1, cb);
        b.record({Ev::Phase, uint8_t(r), 0, uint16_t(k)}, {Strm::Caller, uint8_t(r), 0});
        const StreamId cs{Strm::Copy, uint8_t(r), 0};
        b.wait(cs, {Ev::Phase, uint8_t(r), 0, uint16_t(k)});
        for (int q = 0; q < n; ++q) {
          if (q == r) continue;
          b.touch(cs, q);
          b.ce_copy(cs, recv_at(q, off[r] + rel), own, cb);
        }
      }
      b.plan().sm_bytes += ce[r] * size_t(n - 1);
      b.plan().ce_bytes += ce[r] * size_t(n - 1);
    }
    Loc src[kMaxRanks], dst[kMaxRanks];
    for (int q = 0; q < n; ++q) {
      src[q] = send_at(q, off[r] + ce[r] + host[r]);
      dst[q] = recv_at(q, off[r] + ce[r] + host[r]);
    }
    b.sm_reduce({Strm::Caller, uint8_t(r), 0}, src, n, dst, n, sm);
    b.plan().sm_bytes += sm * size_t(2 * (n - 1));
  }
  for (int r = 0; r < n; ++r) {
    if (!host[r]) continue;
    const size_t base = off[r] + ce[r];
    Loc src[kMaxRanks], dst[kMaxRanks];
    for (int q = 0; q < n; ++q) {
      src[q] = send_at(q, base);
      dst[q] = recv_at(q, base);
    }
    b.host_stage(ranks, src, n, ranks, dst, n, host[r], true);
  }
  if (wrap) b.join();
}

// ReduceScatter: rank r reduces slot r of every rank's input into its output.
void plan_rs_pull(Builder& b, const CliqueDesc& d, const Shares& s) {
  const int n = b.n();
  b.prologue();
  int ranks[kMaxRanks];
  all_ranks(n, ranks);
  const size_t slot = d.bytes;
  const size_t host = n > 1 ? host_share(slot, s.host_ppm, b.policy()) : 0;
  const size_t sm = slot - host;
  for (int r = 0; r < n; ++r) {
    Loc src[kMaxRanks];
    for (int q = 0; q < n; ++q) {
      b.touch({Strm::Caller, uint8_t(r), 0}, q);
      src[q] = send_at(q, size_t(r) * slot);
    }
    Loc dst = recv_at(r, 0);
    b.sm_reduce({Strm::Caller, uint8_t(r), 0}, src, n, &dst, 1, sm);
    b.plan().sm_bytes += sm * size_t(n - 1);
  }
  if (host)
    for (int r = 0; r < n; ++r) {
      Loc src[kMaxRanks];
      for (int q = 0; q < n; ++q) src[q] = send_at(q, size_t(r) * slot + sm);
      Loc dst = recv_at(r, sm);
      b.host_stage(ranks, src, n, &ranks[r], &dst, 1, host, true);
    }
  b.join();
}

// Copy-engine staged AllReduce / ReduceScatter. Rank r owns slice r (AR) or
// slot r (RS). For each piece of it, rank r's copy engine pulls that piece of
// every peer's input into r's scratch (Copy stream); the caller stream folds
// the local input and the staged peer pieces, in rank order, into r's output
// with one local kernel (HBM-bound, fp32 accumulation); for AllReduce the
// Push stream's copy engine then writes the reduced piece into every peer's
// output. Scratch holds `stage_depth` pieces per peer; a piece's scratch is
// refilled only after its fold, and a call's first fill waits for the
// previous staged call's last fold (TempFree). Every NVLink byte moves by
// copy engine, which keeps the link at its bidirectional copy rate.
// Optional host share: the first part of each slice through the host lanes.
void plan_staged(Builder& b, const CliqueDesc& d, const Shares& s, bool allreduce) {
  const int n = b.n();
  b.prologue();
  const Policy& p = b.policy();
  size_t piece = s.stage_piece ? s.stage_piece : p.stage_piece;
  const int depth = s.stage_depth ? s.stage_depth : p.stage_depth;
  int ranks[kMaxRanks];
  all_ranks(n, ranks);
  // A message shorter than one piece stages in pieces of its own (rounded)
  // size, so the scratch it needs scales with the message.
  size_t longest = 0;
  for (int r = 0; r < n; ++r) {
    size_t off = 0, len = d.bytes;
    if (allreduce) slice_of(d.bytes, n, r, &off, &len);
    longest = std::max(longest, len - (n > 1 ? host_share(len, s.host_ppm, p) : 0));
  }
  piece = std::max<size_t>(256, std::min(piece, (longest + 255) / 256 * 256));
  if (n > 1) b.plan().needs.temp_bytes = size_t(depth) * size_t(n - 1) * piece;
  for (int r = 0; r < n; ++r) {
    size_t off, len;
    if (allreduce) {
      slice_of(d.bytes, n, r, &off, &len);
    } else {
      off = size_t(r) * d.bytes;  // source offset of slot r
      len = d.bytes;
    }
    const size_t host = n > 1 ? host_share(len, s.host_ppm, p) : 0;
    const size_t dst_base = allreduce ? off : 0;
    const StreamId cl{Strm::Caller, uint8_t(r), 0};
    const StreamId cs{Strm::Copy, uint8_t(r), 0};
    const StreamId ps{Strm::Push, uint8_t(r), 0};
    int peer_index[kMaxRanks];
    for (int q = 0, j = 0; q < n; ++q) peer_index[q] = q == r ? -1 : j++;
    // The caller stream touches only this rank's buffers and the scratch.
    // The pull stream waits for every peer's input; the push stream's
    // writes into peer outputs are ordered after those waits through the
    // fold it waits for.
    for (int q = 0; q < n; ++q)
      if (q != r) b.touch(cs, q);
    if (allreduce) b.use(ps);
    const size_t staged = len - host;
    int k = 0;
    for (size_t rel = 0; rel < staged; rel += piece, ++k) {
      const size_t cb = std::min(piece, staged - rel);
      const size_t slot = size_t(k % depth) * size_t(n - 1) * piece;
      const size_t src = off + host + rel;
      if (n > 1) {
        if (k >= depth) b.wait(cs, {Ev::Phase, uint8_t(r), 0, uint16_t(2 * (k - depth) + 1)});
        else if (k == 0) b.wait(cs, {Ev::TempFree, uint8_t(r), 0, 0});
        // Peers in rotated order (r+1, r+2, ...): at any moment every rank
        // pulls from a different peer.
        for (int i = 1; i < n; ++i) {
          const int q = (r + i) % n;
          b.ce_copy(cs, temp_at(r, slot + size_t(peer_index[q]) * piece), send_at(q, src), cb);
        }
        b.record({Ev::Phase, uint8_t(r), 0, uint16_t(2 * k)}, cs);
        b.wait(cl, {Ev::Phase, uint8_t(r), 0, uint16_t(2 * k)});
      }
      Loc srcs[kMaxRanks];
      for (int q = 0; q < n; ++q)
        srcs[q] = q == r ? send_at(r, src) : temp_at(r, slot + size_t(peer_index[q]) * piece);
      const Loc dst = recv_at(r, dst_base + host + rel);
      b.sm_reduce(cl, srcs, n, &dst, 1, cb);
      b.record({Ev::Phase, uint8_t(r), 0, uint16_t(2 * k + 1)}, cl);
      if (allreduce && n > 1) {
        b.wait(ps, {Ev::Phase, uint8_t(r), 0, uint16_t(2 * k + 1)});
        for (int i = 1; i < n; ++i)
          b.ce_copy(ps, recv_at((r + i) % n, dst_base + host + rel), dst, cb);
      }
    }
    if (n > 1) b.record({Ev::TempFree, uint8_t(r), 0, 0}, cl);
    b.plan().ce_bytes += staged * size_t(n - 1) * (allreduce ? 2 : 1);
  }
  for (int r = 0; r < n; ++r) {
    size_t off, len;
    if (allreduce) {
      slice_of(d.bytes, n, r, &off, &len);
    } else {
      off = size_t(r) * d.bytes;
      len = d.bytes;
    }
    const size_t host = n > 1 ? host_share(len, s.host_ppm, p) : 0;
    if (!host) continue;
    Loc src[kMaxRanks], dst[kMaxRanks];
    for (int q = 0; q < n; ++q) src[q] = send_at(q, off);
    if (allreduce) {
      for (int q = 0; q < n; ++q) dst[q] = recv_at(q, off);
      b.host_stage(ranks, src, n, ranks, dst, n, host, true);
    } else {
      dst[0] = recv_at(r, 0);
      b.host_stage(ranks, src, n, &ranks[r], dst, 1, host, true);
    }
  }
  b.join();
}

// AllGather: rank r pulls every rank's slot into slot q of its output (its
// own slot too, unless in place). Optional copy-engine and host shares take
// the middle and the suffix of each peer slot.
// push: rank r's kernel stores its own slot into every rank's output (remote
// stores over NVLink) instead of loading every peer's slot (remote loads).
void plan_ag_pull(Builder& b, const CliqueDesc& d, const Shares& s, bool push = false) {
  const int n = b.n();
  b.prologue();
  const size_t slot = d.bytes;
  const size_t host = n > 1 ? host_share(slot, s.host_ppm, b.policy()) : 0;
  const size_t ce = n > 1 ? ce_share(slot - host, s.ce_ppm) : 0;
  const size_t sm = slot - host - ce;
  for (int r = 0; r < n; ++r) {
    Loc dst[kMaxRanks], src[kMaxRanks];
    size_t len[kMaxRanks];
    int k = 0;
    for (int i = 0; i < n; ++i) {
      const int q = push ? (r + i) % n : i;  // pushes start at the own slot, then r+1, r+2, ...
      if (q == r && d.in_place[r]) continue;
      b.touch({Strm::Caller, uint8_t(r), 0}, q);
      dst[k] = push ? recv_at(q, size_t(r) * slot) : recv_at(r, size_t(q) * slot);
      src[k] = push ? send_at(r, 0) : send_at(q, 0);
      // The own slot is a local copy: all of it goes through the SM kernel.
      len[k] = q == r ? slot : sm;
      ++k;
    }
    b.sm_copy({Strm::Caller, uint8_t(r), 0}, dst, src, len, k);
    b.plan().sm_bytes += sm * size_t(n - 1);
    if (ce) {
      // Peers in rotated order (r+1, r+2, ...), alternating between the two
      // copy-engine streams: two engines pull concurrently and, at any
      // moment, no peer serves more than two ranks.
      for (int i = 1; i < n; ++i) {
        const int q = (r + i) % n;
        const StreamId cs{(i % 2) ? Strm::Copy : Strm::Push, uint8_t(r), 0};
        b.touch(cs, r);
        b.touch(cs, q);
        b.ce_copy(cs, recv_at(r, size_t(q) * slot + sm), send_at(q, sm), ce);
      }
      b.plan().ce_bytes += ce * size_t(n - 1);
    }
  }
  if (host)
    for (int q = 0; q < n; ++q) {
      int dst_ranks[kMaxRanks];
      Loc dsts[kMaxRanks];
      int k = 0;
      for (int r = 0; r < n; ++r) {
        if (r == q) continue;
        dst_ranks[k] = r;
        dsts[k++] = recv_at(r, size_t(q) * slot + sm + ce);
      }
      Loc src = send_at(q, sm + ce);
      b.host_stage(&q, &src, 1, dst_ranks, dsts, k, host, false);
    }
  b.join();
}

// Broadcast by pulls: every non-root pulls the root's buffer; the root copies
// its own buffer locally when out of place.
void plan_bc_pull(Builder& b, const CliqueDesc& d, const Shares& s) {
  const int n = b.n();
  const int root = d.root;
  b.prologue();
  const size_t bytes = d.bytes;
  const size_t host = n > 1 ? host_share(bytes, s.host_ppm, b.policy()) : 0;
  const size_t ce = n > 1 ? ce_share(bytes - host, s.ce_ppm) : 0;
  const size_t sm = bytes - host - ce;
  if (!d.in_place[root]) {
    Loc dst = recv_at(root, 0), src = send_at(root, 0);
    b.sm_copy({Strm::Caller, uint8_t(root), 0}, &dst, &src, &bytes, 1);
  }
  for (int r = 0; r < n; ++r) {
    if (r == root) continue;
    b.touch({Strm::Caller, uint8_t(r), 0}, root);
    Loc dst = recv_at(r, 0), src = send_at(root, 0);
    b.sm_copy({Strm::Caller, uint8_t(r), 0}, &dst, &src, &sm, 1);
    b.plan().sm_bytes += sm;
    if (ce) {
      const StreamId cs{Strm::Copy, uint8_t(r), 0};
      b.touch(cs, r);
      b.touch(cs, root);
      b.ce_copy(cs, recv_at(r, sm), send_at(root, sm), ce);
      b.plan().ce_bytes += ce;
    }
  }
  if (host) {
    int dst_ranks[kMaxRanks];
    Loc dsts[kMaxRanks];
    int k = 0;
    for (int r = 0; r < n; ++r) {
      if (r == root) continue;
      dst_ranks[k] = r;
      dsts[k++] = recv_at(r, sm + ce);
    }
    Loc src = send_at(root, sm + ce);
    b.host_stage(&root, &src, 1, dst_ranks, dsts, k, host, false);
  }
  b.join();
}

// Broadcast by scatter + all-gather over the N-1 non-roots, in pipelined
// pieces. Phase 1 (caller stream): non-root j pulls its slice of the piece
// from the root. Phase 2 (aux stream): after every other non-root's phase 1
// of that piece, non-root j pulls the other slices from their owners. The
// root sends each byte once and every non-root receives each byte once.
void plan_bc_scatter(Builder& b, const CliqueDesc& d, const Shares& s) {
  const int n = b.n();
  const int root = d.root;
  b.prologue();
  const size_t bytes = d.bytes;
  const size_t host = host_share(bytes, s.host_ppm, b.policy());
  const size_t body = bytes - host;
  int nonroot[kMaxRanks];
  int m = 0;
  for (int r = 0; r < n; ++r)
    if (r != root) nonroot[m++] = r;
  const size_t min_piece = 16 * kMiB;
  int pieces = std::max(1, b.policy().bc_pieces);
  while (pieces > 1 && body / size_t(pieces) < min_piece) --pieces;
  // With a copy-engine share every byte moves by copy engine: phase 1 on the
  // Copy stream, phase 2 on the Push stream; otherwise by SM copy kernels on
  // the caller and aux streams.
  const bool ce = s.ce_ppm >= 5000;
  auto phase1 = [&](int r) -> StreamId { return {ce ? Strm::Copy : Strm::Caller, uint8_t(r), 0}; };
  auto phase2 = [&](int r) -> StreamId { return {ce ? Strm::Push : Strm::Aux, uint8_t(r), 0}; };
  size_t& moved = ce ? b.plan().ce_bytes : b.plan().sm_bytes;
  if (!d.in_place[root]) {
    const StreamId as = phase2(root);
    b.touch(as, root);
    Loc dst = recv_at(root, 0), src = send_at(root, 0);
    if (ce) b.ce_copy(as, dst, src, bytes);
    else b.sm_copy(as, &dst, &src, &bytes, 1);
  }
  for (int k = 0; k < pieces; ++k) {
    size_t poff, plen;
    slice_of(body, pieces, k, &poff, &plen);
    for (int j = 0; j < m; ++j) {
      size_t soff, slen;
      slice_of(plen, m, j, &soff, &slen);
      const int r = nonroot[j];
      const StreamId s1 = phase1(r);
      b.touch(s1, root);
      b.touch(s1, r);
      Loc dst = recv_at(r, poff + soff), src = send_at(root, poff + soff);
      if (ce) b.ce_copy(s1, dst, src, slen);
      else b.sm_copy(s1, &dst, &src, &slen, 1);
      b.record({Ev::Phase, uint8_t(r), 0, uint16_t(k)}, s1);
      moved += slen;
    }
    for (int j = 0; j < m; ++j) {
      const int r = nonroot[j];
      const StreamId as = phase2(r);
      b.touch(as, r);
      Loc dst[kMaxRanks], src[kMaxRanks];
      size_t len[kMaxRanks];
      int c = 0;
      for (int t = 1; t < m; ++t) {  // rotated: non-root j reads j+1, j+2, ...
        const int i = (j + t) % m;
        const int q = nonroot[i];
        b.wait(as, {Ev::Phase, uint8_t(q), 0, uint16_t(k)});
        size_t soff, slen;
        slice_of(plen, m, i, &soff, &slen);
        dst[c] = recv_at(r, poff + soff);
        src[c] = recv_at(q, poff + soff);
        len[c++] = slen;
        moved += slen;
      }
      if (ce)
        for (int i = 0; i < c; ++i) b.ce_copy(as, dst[i], src[i], len[i]);
      else
        b.sm_copy(as, dst, src, len, c);
    }
  }
  if (host) {
    Loc dsts[kMaxRanks];
    for (int j = 0; j < m; ++j) dsts[j] = recv_at(nonroot[j], body);
    Loc src = send_at(root, body);
    b.host_stage(&root, &src, 1, nonroot, dsts, m, host, false);
  }
  b.join();
}

// Broadcast by a pipelined chain over the ranks root, root+1, ..., root+n-1.
// The buffer is cut into pieces; hop h (1..n-1) pulls piece k from hop h-1
// (the root's send buffer for h = 1, else the predecessor's output) once the
// predecessor holds it. Every rank receives each byte once and forwards it
// once, so every link carries the buffer once per direction and the hops of
// different pieces overlap; the time is about (pieces + n - 2) piece times.
// Data moves by copy engine (ce share >= 50 %) or by SM copy kernels.
void plan_bc_chain(Builder& b, const CliqueDesc& d, const Shares& s) {
  const int n = b.n();
  const int root = d.root;
  b.prologue();
  const Policy& p = b.policy();
  const size_t bytes = d.bytes;
  const size_t host = n > 1 ? host_share(bytes, s.host_ppm, p) : 0;
  const size_t body = bytes - host;
  const size_t piece = s.stage_piece ? s.stage_piece : p.stage_piece;
  const bool ce = s.ce_ppm >= 5000;
  size_t& moved = ce ? b.plan().ce_bytes : b.plan().sm_bytes;
  if (!d.in_place[root]) {
    const StreamId as{ce ? Strm::Push : Strm::Aux, uint8_t(root), 0};
    b.touch(as, root);
    const Loc dst = recv_at(root, 0), src = send_at(root, 0);
    if (ce) b.ce_copy(as, dst, src, bytes);
    else b.sm_copy(as, &dst, &src, &bytes, 1);
  }
  int k = 0;
  for (size_t off = 0; off < body; off += piece, ++k) {
    const size_t cb = std::min(piece, body - off);
    for (int h = 1; h < n; ++h) {
      const int r = (root + h) % n, pred = (root + h - 1) % n;
      // Copy-engine pieces alternate between two streams of the receiver, so
      // the next piece's copy is queued while the previous one drains.
      const StreamId s1{ce ? (k % 2 ? Strm::Push : Strm::Copy) : Strm::Caller, uint8_t(r), 0};
      b.touch(s1, r);
      b.touch(s1, pred);
      if (h > 1) b.wait(s1, {Ev::Phase, uint8_t(pred), 0, uint16_t(k)});
      const Loc src = h == 1 ? send_at(root, off) : recv_at(pred, off);
      const Loc dst = recv_at(r, off);
      if (ce) b.ce_copy(s1, dst, src, cb);
      else b.sm_copy(s1, &dst, &src, &cb, 1);
      b.record({Ev::Phase, uint8_t(r), 0, uint16_t(k)}, s1);
      moved += cb;
    }
  }
  if (host) {
    int nonroot[kMaxRanks];
    Loc dsts[kMaxRanks];
    int m = 0;
    for (int r = 0; r < n; ++r)
      if (r != root) {
        nonroot[m] = r;
        dsts[m++] = recv_at(r, body);
      }
    const Loc src = send_at(root, body);
    b.host_stage(&root, &src, 1, nonroot, dsts, m, host, false);
  }
  b.join();
}

// NVLS routes (AllReduce, Broadcast, AllGather, ReduceScatter): one gang op
// per rank on its aux stream, after every rank's input is ready. Inside,
// the kernels move data through the rank's multicast-bound scratch and the
// switch (multimem.ld_reduce / multimem.st) with bounded in-kernel barriers
// between pipelined rounds (exec/nvls.cu). The prologue waits make the
// members of a gang start together, so those barriers wait only for skew.
void plan_ar_nvls(Builder& b, const CliqueDesc& d, const Policy& p, const Shares& s) {
  const int n = b.n();
  b.prologue();
  for (int r = 0; r < n; ++r) {
    const StreamId as{Strm::Aux, uint8_t(r), 0};
    for (int q = 0; q < n; ++q) b.touch(as, q);
    b.nvls(as, r, d.bytes);
    PlanOp& op = b.plan().ops.back();
    op.nvls_movers = uint16_t(std::max(0, s.nvls_movers));
    op.nvls_unroll = uint8_t(std::max(0, s.nvls_unroll));
    op.nvls_round = size_t(std::max(0, s.nvls_round_mib)) << 20;
    op.nvls_ramp = uint8_t(std::clamp(s.nvls_ramp, 0, 2));
    op.nvls_ahead = uint8_t(std::clamp(s.nvls_ahead, 0, 2));
  }
  b.plan().needs.nvls_bytes = p.nvls_round_bytes;
  b.plan().sm_bytes += d.bytes * size_t(n);  // ~S in and S out per GPU via the switch
  b.join();
}

// Broadcast push chain (exec/ring.cu): one gang op per rank on its caller
// stream after every rank's input is ready; inside, each rank forwards
// pieces to its successor as they arrive (in-kernel progress words).
void plan_bc_ring(Builder& b, const CliqueDesc& d) {
  const int n = b.n();
  b.gang_fence();
  b.prologue();
  for (int r = 0; r < n; ++r) {
    const StreamId cs{Strm::Caller, uint8_t(r), 0};
    for (int q = 0; q < n; ++q) b.touch(cs, q);
    b.nvls(cs, r, d.bytes);
    b.gang_done(r);
  }
  b.plan().needs.ring = true;
  b.plan().sm_bytes += d.bytes * size_t(n - 1);
  b.join();
}

// Hybrid AllReduce: the first share of the message through the switch (an
// NVLS gang on `hybrid_blocks` SMs per GPU, launched first), the rest by the
// two-shot P2P kernel, which the remaining SMs run at the same time; both
// shares cross NVLink concurrently. The split point is 4 KiB aligned. The
// gate refuses the hybrid routes (wrong data at 4 GiB on the GPU, slower
// than NVLS alone where correct); the planners stay for the plan checks.
int split_ppm(const Policy& p, const Shares& s) { return s.split_ppm > 0 ? s.split_ppm : p.hybrid_nvls_ppm; }
uint16_t split_blocks(const Policy& p, const Shares& s) {
  return uint16_t(s.split_blocks > 0 ? s.split_blocks : p.hybrid_blocks);
}

void plan_ar_hybrid(Builder& b, const CliqueDesc& d, const Policy& p, const Shares& s) {
  const int n = b.n();
  b.prologue();
  const size_t nv = d.bytes / 10000 * size_t(split_ppm(p, s)) / 4096 * 4096;
  for (int r = 0; r < n; ++r) {
    const StreamId as{Strm::Aux, uint8_t(r), 0};
    for (int q = 0; q < n; ++q) b.touch(as, q);
    if (nv) b.nvls(as, r, nv, 0, split_blocks(p, s));
  }
  if (nv) {
    b.plan().needs.nvls_bytes = p.nvls_round_bytes;
    b.plan().sm_bytes += nv * size_t(n);
  }
  Shares none = s;
  none.host_ppm = none.ce_ppm = 0;
  plan_ar_twoshot(b, d, none, nv, d.bytes - nv, false);
  b.join();
}

// Hybrid ReduceScatter: the leading share of every slot through the switch
// (the NVLS ReduceScatter gang on part of the SMs, launched first on the aux
// streams), the rest of each slot by the P2P pull fold on the caller
// streams, at the same time. NVLS reads every slot of every GPU once through
// the switch while the pulls use the links' remaining capacity.
void plan_rs_hybrid(Builder& b, const CliqueDesc& d, const Policy& p, const Shares& s) {
  const int n = b.n();
  b.prologue();
  const size_t slot = d.bytes;
  const size_t nv = slot / 10000 * size_t(split_ppm(p, s)) / 4096 * 4096;
  for (int r = 0; r < n; ++r) {
    const StreamId as{Strm::Aux, uint8_t(r), 0};
    for (int q = 0; q < n; ++q) b.touch(as, q);
    if (nv) b.nvls(as, r, nv, 0, split_blocks(p, s));
  }
  if (nv) {
    b.plan().needs.nvls_bytes = p.nvls_round_bytes;
    b.plan().sm_bytes += nv * size_t(n) * size_t(n);
  }
  for (int r = 0; r < n && nv < slot; ++r) {
    const StreamId cs{Strm::Caller, uint8_t(r), 0};
    Loc src[kMaxRanks];
    for (int q = 0; q < n; ++q) {
      b.touch(cs, q);
      src[q] = send_at(q, size_t(r) * slot + nv);
    }
    const Loc dst = recv_at(r, nv);
    b.sm_reduce(cs, src, n, &dst, 1, slot - nv);
    b.plan().sm_bytes += (slot - nv) * size_t(n - 1);
  }
  b.join();
}

// Push-reduce ReduceScatter / AllReduce (exec/pushred.cu): one gang op per
// rank on its caller stream after every rank's input is ready.
void plan_pushred(Builder& b, const CliqueDesc& d) {
  const int n = b.n();
  b.gang_fence();
  b.prologue();
  for (int r = 0; r < n; ++r) {
    const StreamId cs{Strm::Caller, uint8_t(r), 0};
    for (int q = 0; q < n; ++q) b.touch(cs, q);
    b.nvls(cs, r, d.bytes);
    b.gang_done(r);
  }
  b.plan().needs.pushred = true;
  const size_t moved = d.kind == Kind::AllReduce ? d.bytes * size_t(2 * (n - 1)) : d.bytes * size_t(n - 1) * size_t(n);
  b.plan().sm_bytes += moved;
  b.join();
}

// AllReduce one-shot (exec/oneshot.cu): one gang op per rank on its caller
// stream and nothing else -- no event records or waits. Inside, every
// rank's blocks meet their counterparts on every GPU (arrive), fold the
// whole message from all N inputs in rank order into their own output only,
// and meet again (depart) before the stream may go on. Each GPU reads
// (N-1) x S over NVLink, so the route pays for small and medium messages,
// where the cross-device event fans of an event-ordered plan would cost
// more than the bytes. In place, a rank would overwrite its input while
// peers still read it, so an in-place call takes the two-shot plan instead.
void plan_ar_oneshot(Builder& b, const CliqueDesc& d) {
  const int n = b.n();
  for (int r = 0; r < n; ++r) b.nvls({Strm::Caller, uint8_t(r), 0}, r, d.bytes);
  b.plan().needs.oneshot = true;
  b.plan().sm_bytes += d.bytes * size_t(n - 1) * size_t(n);
}

// Low-latency two-shot AllReduce (exec/oneshot.cu, two-shot mode): the same
// gang kernel per rank on its caller stream and no events; rank r folds
// slice r from every input and stores it into every rank's output, between
// the in-kernel arrive and depart barriers. In place is safe: each element
// of slice r is read and written by the same thread of rank r only.
void plan_ar_twoshot_ll(Builder& b, const CliqueDesc& d) {
  const int n = b.n();
  for (int r = 0; r < n; ++r) {
    size_t off, len;
    slice_of(d.bytes, n, r, &off, &len);
    b.nvls({Strm::Caller, uint8_t(r), 0}, r, len, off);
  }
  b.plan().needs.oneshot = true;
  b.plan().sm_bytes += d.bytes * size_t(2 * (n - 1));
}

// Low-latency ReduceScatter / AllGather / Broadcast on the one-shot engine:
// one gang kernel per rank on its caller stream, no events. Rank r folds
// slot r from every input into its output (ReduceScatter), stores its slot
// into slot r of every rank's output (AllGather), or copies the root's
// buffer into its output (Broadcast), between the in-kernel arrive and
// depart barriers. Counterparts: the reference's event-ordered copy-engine
// copies of the peer's slot (shim/nccl_collectives_shim.cu:626) and of the
// root's buffer (:674), for two GPUs.
void plan_gang_ll(Builder& b, const CliqueDesc& d) {
  const int n = b.n();
  for (int r = 0; r < n; ++r) b.nvls({Strm::Caller, uint8_t(r), 0}, r, d.bytes);
  b.plan().needs.oneshot = true;
  // NVLink bytes: every non-root reads the root's buffer (Broadcast); every
  // rank moves its slot to or from each peer (AllGather, ReduceScatter).
  b.plan().sm_bytes += d.bytes * size_t(n - 1) * (d.kind == Kind::Broadcast ? 1 : size_t(n));
}

// One rank: every collective except a scaled one (PreMulSum) is a copy of
// the input into the output: the SM stream copy kernel on the caller stream,
// beside an optional copy-engine share (the leading ce_ppm of the bytes, on
// the copy stream) that the init-time tuning keeps when the two engines
// together move more than the kernel alone.
void plan_single(Builder& b, const CliqueDesc& d, const Shares& s) {
  b.prologue();
  const StreamId cl{Strm::Caller, 0, 0};
  b.touch(cl, 0);
  if (!d.in_place[0]) {
    const size_t ce = ce_share(d.bytes, s.ce_ppm) & ~size_t(31);  // keeps the SM part 32-byte aligned
    if (ce) {
      const StreamId cp{Strm::Copy, 0, 0};
      b.touch(cp, 0);
      b.ce_copy(cp, recv_at(0, 0), send_at(0, 0), ce);
    }
    const Loc dst = recv_at(0, ce), src = send_at(0, ce);
    const size_t len = d.bytes - ce;
    b.sm_copy(cl, &dst, &src, &len, 1);
  }
  b.join();
}

}  // namespace

void build_plan(Algo algo, const CliqueDesc& d, const Policy& p, const Shares& s, Plan& out) {
  Builder b(out, algo, d, p);
  if (d.nranks == 1 && algo != Algo::Fallback && !(reduces(d.kind) && d.op == RedOp::PreMulSum)) {
    plan_single(b, d, s);
    return;
  }
  bool in_place = false;
  for (int r = 0; r < d.nranks; ++r) in_place = in_place || d.in_place[r];
  if (algo == Algo::ArOneShot && in_place) algo = Algo::ArTwoShotLL;
  b.plan().algo = algo;
  switch (algo) {
    case Algo::ArOneShot: plan_ar_oneshot(b, d); break;
    case Algo::ArTwoShotLL: plan_ar_twoshot_ll(b, d); break;
    case Algo::RsLL: case Algo::AgLL: case Algo::BcLL: plan_gang_ll(b, d); break;
    case Algo::ArTwoShot: plan_ar_twoshot(b, d, s); break;
    case Algo::ArNvls: plan_ar_nvls(b, d, p, s); break;
    case Algo::RsPull: plan_rs_pull(b, d, s); break;
    case Algo::AgPull: plan_ag_pull(b, d, s); break;
    case Algo::AgPush: plan_ag_pull(b, d, s, true); break;
    case Algo::BcRing: plan_bc_ring(b, d); break;
    case Algo::RsPush: case Algo::ArPush: plan_pushred(b, d); break;
    case Algo::ArHybrid: plan_ar_hybrid(b, d, p, s); break;
    case Algo::RsHybrid: plan_rs_hybrid(b, d, p, s); break;
    case Algo::BcPull: plan_bc_pull(b, d, s); break;
    case Algo::BcScatter: plan_bc_scatter(b, d, s); break;
    case Algo::ArStaged: plan_staged(b, d, s, true); break;
    case Algo::RsStaged: plan_staged(b, d, s, false); break;
    case Algo::BcChain: plan_bc_chain(b, d, s); break;
    case Algo::BcNvls: case Algo::AgNvls: case Algo::RsNvls: plan_ar_nvls(b, d, p, s); break;
    default: break;
  }
}

Needs prewarm_needs(int nranks, const Policy& p, const Shares& s, bool nvls) {
  Needs needs;
  if (s.host_ppm > 0) {
    needs.lanes = p.lanes;
    needs.bounce_bytes = p.host_piece;
  }
  needs.phase_events = uint16_t(std::max(64, p.bc_pieces));
  if (nvls && nranks >= 2) needs.nvls_bytes = p.nvls_round_bytes;
  return needs;
}

}  // namespace nb
