// The plan submission loop and its error classification, independent of
// CUDA so the error policy can be tested on the CPU with a fake submitter.
//
// Every op is submitted in plan order. A failure before any data op (copy,
// kernel, host task) was attempted is NotStarted: only event records/waits
// reached the streams, which order but never touch data, so NCCL may still
// run the call. A failure of the first data op or any later op is Failed.
// The fault injector can make any op fail without calling the submitter.
//
// Parity: execute_plan of the reference (shim/nccl_collectives_shim.cu:
// 1168-1194).
#pragma once

#include <cstddef>

#include "core/fault.h"
#include "core/plan.h"

namespace nb {

enum class ExecStatus { Ok, NotStarted, Failed };

inline bool is_data_op(OpKind k) { return k != OpKind::Record && k != OpKind::Wait; }

// submit(op, index) returns 0 on success or an error code. On failure,
// *error gets the code (or `injected_error` for an injected fault) and
// *failed_at the op index.
template <typename Submit>
ExecStatus run_plan_ops(const Plan& plan, Submit&& submit, FaultInjector* fault, int injected_error,
                        int* error, size_t* failed_at) {
  bool started = false;
  for (size_t i = 0; i < plan.ops.size(); ++i) {
    const PlanOp& op = plan.ops[i];
    // An attempted data op counts as started even when it fails: it may have
    // been partly enqueued.
    started |= is_data_op(op.kind);
    const int e = (fault && fault->fail_op(i)) ? injected_error  // nothing is submitted
                                               : submit(op, i);
    if (e != 0) {
      if (error) *error = e;
      if (failed_at) *failed_at = i;
      return started ? ExecStatus::Failed : ExecStatus::NotStarted;
    }
  }
  return ExecStatus::Ok;
}

}  // namespace nb
