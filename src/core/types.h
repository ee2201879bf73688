// Pure type model of the interposer: collective kinds, element types,
// reduction operators, algorithms and fallback reasons, plus the per-call
// descriptor and its buffer geometry. No CUDA, no NCCL header: NCCL enum
// values are carried as plain ints (their numeric values are NCCL ABI).
//
// Parity: the reference's Layer-2 type model (shim/nccl_collectives_shim.cu:107-176)
// covers two ranks, sum only and fp32/fp16/bf16 reductions. This model covers
// 1..8 ranks of one clique, sum/prod/max/min/avg/premulsum and every NCCL
// reducible type the kernels implement.
#pragma once

#include <cstddef>
#include <cstdint>

namespace nb {

constexpr size_t kMiB = size_t(1) << 20;
constexpr size_t kGiB = size_t(1) << 30;
constexpr int kMaxRanks = 8;
constexpr int kMaxLanes = 8;

// NCCL ABI values (nccl.h); kept here so the pure core needs no NCCL header.
namespace nccl {
constexpr int Success = 0, UnhandledCudaError = 1, SystemError = 2, InternalError = 3,
              InvalidArgument = 4, InvalidUsage = 5;
constexpr int Int8 = 0, Uint8 = 1, Int32 = 2, Uint32 = 3, Int64 = 4, Uint64 = 5, Float16 = 6,
              Float32 = 7, Float64 = 8, Bfloat16 = 9, Float8e4m3 = 10, Float8e5m2 = 11;
constexpr int Sum = 0, Prod = 1, Max = 2, Min = 3, Avg = 4, NumOps = 5;
}  // namespace nccl

enum class Kind : uint8_t { AllReduce, AllGather, ReduceScatter, Broadcast, Count };
enum class DType : uint8_t { Unsupported, I8, U8, I32, U32, I64, U64, F16, F32, F64, BF16, F8E4M3, F8E5M2, Count };
// PreMulSum is a user-created op (ncclRedOpCreatePreMulSum) learned by the
// interposer; Unsupported covers unknown dynamic ops.
enum class RedOp : uint8_t { Sum, Prod, Max, Min, Avg, PreMulSum, Unsupported, Count };

// Algorithms the planner can pick. Fallback means "libnccl runs it".
enum class Algo : uint8_t {
  Fallback,
  ArTwoShot,   // rank r reduces slice r from every peer and pushes it to every peer
  ArNvls,      // multimem.ld_reduce / multimem.st through the NVSwitch
  RsPull,      // rank r reduces slot r from every peer into its own output
  AgPull,      // rank r pulls every peer's slot into its own output
  BcPull,      // every non-root pulls the root's buffer (2 ranks)
  BcScatter,   // scatter slices from the root, then all-gather them (N ranks)
  ArStaged,    // copy engines pull slice r into scratch, a local fused fold, CE pushes
  RsStaged,    // copy engines pull slot r into scratch, a local fused fold
  BcChain,     // pipelined chain: each rank pulls every piece from its predecessor
  BcNvls,      // the root multicasts through the switch (multimem.st)
  AgNvls,      // every rank multicasts its slot through the switch
  RsNvls,      // every rank multimem.ld_reduces its own slot
  AgPush,      // every rank stores its slot into every rank's output
  BcRing,      // pipelined push chain with in-kernel progress words
  RsPush,      // senders store into owners' scratch; owners fold (stores only)
  ArPush,      // RsPush, then owners store the result into every output
  ArHybrid,    // NVLS on part of the SMs for one share, two-shot P2P for the rest
  ArOneShot,   // every rank folds the whole message from all inputs into its own output
  RsHybrid,    // NVLS ReduceScatter on part of the SMs for one share, P2P pulls for the rest
  ArTwoShotLL, // two-shot in one gang kernel per rank: in-kernel arrive/depart instead of events
  RsLL,        // ReduceScatter fold of slot r in one gang kernel per rank (arrive/depart)
  AgLL,        // AllGather: each rank stores its slot into every output (arrive/depart)
  BcLL,        // Broadcast: each rank copies the root's buffer (arrive/depart)
  Count
};

enum class Reason : uint8_t {
  None, NotGrouped, UnsupportedType, UnsupportedOp, NullBuffer, SizeOverflow,
  BelowThreshold, Misaligned, BadSlot, PartialOverlap, BadRank, GroupShape,
  NotClique, Mismatch, Capturing, FirstPass, SetupFailed, SubmitFailedEarly,
  Poisoned, AboveLimit, AddressOverflow, PolicyFallback, MetadataQuery,
  RuntimeUnsupported, UnsupportedNccl, Disabled, FaultInjected, DeviceTimeout,
  Count
};

const char* kind_name(Kind k);
const char* dtype_name(DType t);
const char* op_name(RedOp o);
const char* algo_name(Algo a);
const char* reason_name(Reason r);

size_t elem_size(DType t);
// Types the reduction kernels implement (sum/prod/max/min for all of them;
// avg and premulsum for the floating types only).
bool reducible(DType t);
bool is_float(DType t);
DType dtype_from_nccl(int nccl_type);
int dtype_to_nccl(DType t);

// One intercepted collective call. `count` follows NCCL: AllGather send
// count, ReduceScatter receive count, element count otherwise.
struct CallDesc {
  Kind kind = Kind::AllReduce;
  DType dtype = DType::Unsupported;
  RedOp op = RedOp::Sum;
  size_t count = 0;
  uintptr_t send = 0, recv = 0;
  int device = -1, rank = -1, nranks = -1, root = -1;
  // PreMulSum scalar (per rank, as NCCL defines it). residence 1 = host
  // immediate (value captured in `scalar`), 0 = device pointer.
  int scalar_residence = 1;
  double scalar = 1.0;
  uintptr_t scalar_ptr = 0;
};

bool reduces(Kind k);
// Per-rank payload in bytes: the AllReduce/Broadcast buffer, the AllGather
// send slot or the ReduceScatter receive slot.
size_t call_bytes(const CallDesc& c);
size_t send_extent(const CallDesc& c);
size_t recv_extent(const CallDesc& c);
// The whole logical message (nccl-tests "size"): N slots for AG/RS.
size_t logical_bytes(const CallDesc& c);
// The in-place layouts NCCL defines; any other send/recv overlap falls back.
bool call_in_place(const CallDesc& c);
inline bool ranges_overlap(uintptr_t a, size_t an, uintptr_t b, size_t bn) {
  return a < b + bn && b < a + an;
}

}  // namespace nb
