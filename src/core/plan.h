// Pure schedule IR and the per-algorithm planners.
//
// A Plan is an ordered list of ops on logical streams (per rank: the
// caller's stream, an auxiliary SM stream, a copy-engine stream, per-lane
// D2H/H2D streams; per lane: a host-reduction stream), ordered across streams
// by logical events. The executor binds streams, events and buffers and
// submits the ops in order; the CPU simulator (plan_sim.h) runs the same
// plans on host memory and checks every conflicting access pair for a
// happens-before edge.
//
// Parity: the reference's Layer-3 IR (shim/nccl_collectives_shim.cu:292-418:
// Record/Wait/Copy/Reduce on Caller/Copy/HostReduce/Side/D2H/H2D streams) and
// its route builders (:420-714). Differences: N ranks instead of a device
// pair; a data op is a fused multi-source reduce or multi-segment copy that
// one sm_100a kernel performs while moving the bytes over NVLink (no Temp
// scratch round-trip); the host lane reduces on the CPU.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include "core/gate.h"
#include "core/policy.h"
#include "core/types.h"

namespace nb {

// Logical streams. `dev` is a rank index of the clique. D2H and H2D lanes
// live on rank `dev`'s GPU; Host(lane) lives on rank 0's GPU and only waits,
// records and runs the CPU reduction.
// Copy and Push are two copy-engine streams per GPU (pulls and pushes of a
// staged route run concurrently on different engines).
// Hub is one stream on rank 0's GPU that gathers the ranks' readiness and
// completion for cliques of four or more (see Builder::prologue/join).
enum class Strm : uint8_t { Caller, Aux, Copy, D2H, H2D, Host, Push, Hub, Count };
struct StreamId {
  Strm kind = Strm::Caller;
  uint8_t dev = 0;
  uint8_t lane = 0;
};
bool operator==(StreamId a, StreamId b);
inline bool operator!=(StreamId a, StreamId b) { return !(a == b); }

// Logical events, each recorded on one stream. Done(stream) marks the end of
// an internal stream's work in this plan (index = stream kind).
// TempFree(dev) marks the end of a staged call's last read of its scratch:
// the next staged call's first copy into that scratch waits for it.
// GangDone(dev) marks the end of the last gang op a caller stream ran on that
// GPU (push chain, push-reduce): those engines keep per-device-set scratch,
// progress words and an epoch, so the next such call waits for GangDone on
// every GPU of its clique before it starts (two calls on unordered streams,
// or from two cliques over the same GPUs, never overlap).
// AllReady / AllJoined are recorded on the hub once it has waited for every
// rank's InputReady / Join.
enum class Ev : uint8_t { InputReady, Join, Phase, Done, D2HDone, H2DDone, HostDone, LaneFree, TempFree,
                          GangDone, AllReady, AllJoined, Count };
struct EventId {
  Ev kind = Ev::InputReady;
  uint8_t dev = 0;
  uint8_t lane = 0;
  uint16_t index = 0;
};
bool operator==(EventId a, EventId b);

// Buffers. Send/Recv are the caller's (per rank); Bounce(dev, lane) is the
// pinned-host staging buffer a rank's D2H fills; HostOut(lane) holds the
// host reduction's result.
// Temp(dev) is a per-GPU device scratch buffer the staged routes land peer
// data in.
enum class Buf : uint8_t { None, Send, Recv, Bounce, HostOut, Temp };
struct Loc {
  Buf buf = Buf::None;
  uint8_t dev = 0;
  uint8_t lane = 0;
  size_t off = 0;
};
inline Loc at(Loc l, size_t by) { l.off += by; return l; }
inline Loc send_at(int r, size_t off) { return {Buf::Send, uint8_t(r), 0, off}; }
inline Loc recv_at(int r, size_t off) { return {Buf::Recv, uint8_t(r), 0, off}; }
inline Loc bounce_at(int r, int lane) { return {Buf::Bounce, uint8_t(r), uint8_t(lane), 0}; }
inline Loc hostout_at(int lane) { return {Buf::HostOut, 0, uint8_t(lane), 0}; }
inline Loc temp_at(int r, size_t off) { return {Buf::Temp, uint8_t(r), 0, off}; }

// Record: event := current position of stream.   Wait: stream waits event.
// CeCopy: dst[0,bytes) := src[0,bytes) by a copy engine.
// SmCopy: for each segment i, dst[i][0,len[i]) := src[i][0,len[i]), one kernel.
// SmReduce: v := op-fold of src[0..nsrc) in index order; every dst[j] := v.
// HostReduce: the same fold on the CPU over pinned-host buffers.
// NvlsReduce: one rank's share of a gang collective (NVLS, push chain,
// push-reduce); the N NvlsReduce ops of a plan form a gang that synchronizes
// inside the kernel. For AllReduce it covers [src[0].off, +bytes) of every
// rank's buffers; for ReduceScatter that range of every slot; for the other
// kinds the whole message.
enum class OpKind : uint8_t { Record, Wait, CeCopy, SmCopy, SmReduce, HostReduce, NvlsReduce };
struct PlanOp {
  OpKind kind = OpKind::Record;
  StreamId stream;
  EventId event;
  uint8_t nsrc = 0, ndst = 0;
  Loc src[kMaxRanks];
  Loc dst[kMaxRanks];
  size_t len[kMaxRanks] = {};
  size_t bytes = 0;
  uint16_t grid = 0;  // gang ops: blocks per GPU (0 = one per SM)
  // NVLS gang ops: the kernel's shape (0 = the policy's): switch-side
  // threads per block, multimem requests in flight per thread, round bytes,
  // AllReduce round schedule (1 uniform, 2 ramped).
  uint16_t nvls_movers = 0;
  uint8_t nvls_unroll = 0;
  uint8_t nvls_ramp = 0;
  uint8_t nvls_ahead = 0;  // AllReduce copier: 1 usual order, 2 every copy-in first
  size_t nvls_round = 0;
};

// Resources a plan needs; the executor allocates them before submitting.
struct Needs {
  int lanes = 0;               // host lanes used
  size_t bounce_bytes = 0;     // per rank per lane, and per HostOut lane
  uint16_t phase_events = 0;   // Phase(dev, index) indices per rank
  size_t nvls_bytes = 0;       // multicast scratch per GPU
  size_t temp_bytes = 0;       // device scratch per GPU (staged routes)
  bool ring = false;           // progress words for the in-kernel chain
  bool pushred = false;        // scratch and progress words of the push-reduce engine
  bool oneshot = false;        // arrive/depart tables of the one-shot engine
  void merge(const Needs& o);
};

// Per-path shares in parts per 10000 of the bytes a rank receives.
// Staged routes also take their pipeline shape from here (0 = policy default).
struct Shares {
  int host_ppm = 0;
  int ce_ppm = 0;
  size_t stage_piece = 0;
  int stage_depth = 0;
  // Hybrid routes: the switch's share of the message (per 10000) and the
  // blocks per GPU its kernel gets (0 = the policy's).
  int split_ppm = 0;
  int split_blocks = 0;
  // NVLS routes: the kernel shape (0 = the policy's).
  int nvls_movers = 0;
  int nvls_unroll = 0;
  int nvls_round_mib = 0;
  int nvls_ramp = 0;  // 0 = the policy's, 1 = uniform rounds, 2 = ramped
  int nvls_ahead = 0;  // 0 = the policy's, 1 = usual copier order, 2 = every copy-in first
};

struct Plan {
  Algo algo = Algo::Fallback;
  CliqueDesc desc;
  std::vector<PlanOp> ops;
  Needs needs;
  // Byte accounting per path (summed over ranks): what crossed NVLink by SM
  // kernels, by copy engines, and through pinned host memory.
  size_t sm_bytes = 0, ce_bytes = 0, host_bytes = 0;
};

// 32-byte-aligned split of `bytes` into `parts` consecutive slices (the
// kernels' widest vector); the last slice takes the remainder.
void slice_of(size_t bytes, int parts, int i, size_t* off, size_t* len);
// Host-lane share of `len` bytes at `ppm`: a whole number of 16-byte units,
// zero below the policy minimum.
size_t host_share(size_t len, int ppm, const Policy& p);
size_t ce_share(size_t len, int ppm);

void build_plan(Algo algo, const CliqueDesc& d, const Policy& p, const Shares& s, Plan& out);

// Resources for the largest call the prewarm covers (at InitAll).
Needs prewarm_needs(int nranks, const Policy& p, const Shares& s, bool nvls);

}  // namespace nb
