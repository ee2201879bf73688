// Host-side fault injector. It makes one plan submission step report a CUDA
// error code WITHOUT calling CUDA, so both error policies can be exercised
// on a CPU or on a GPU with nothing faulting:
//   setup         the resource setup of the next custom call fails
//                 -> the call falls back to NCCL (SetupFailed);
//   op:K          the K-th submitted op of the next custom call fails; if no
//                 copy or kernel was submitted before it, the call falls back
//                 (SubmitFailedEarly), otherwise the process is poisoned and
//                 the call returns ncclUnhandledCudaError.
// Spec (NCCL_B200_FAULT): "setup", "op:K", optionally followed by ":always"
// (fire on every custom call, not only the first).
//
// Parity: the reference has no injector; its stress harness only expects an
// error it cannot produce (tests/stress_check.cu:1034-1048).
#pragma once

#include <atomic>
#include <string>

namespace nb {

class FaultInjector {
 public:
  bool configure(const std::string& spec);
  bool active() const { return kind_ != Kind::None; }
  // Called once per custom call, before setup.
  bool fail_setup();
  // Called per submitted op (0-based index within the call).
  bool fail_op(size_t index);
  // Called after a call finishes submission (one-shot faults disarm).
  void end_call();

 private:
  enum class Kind { None, Setup, Op };
  Kind kind_ = Kind::None;
  size_t index_ = 0;
  bool always_ = false;
  std::atomic<bool> fired_{false};
};

}  // namespace nb
