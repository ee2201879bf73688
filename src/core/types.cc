#include "core/types.h"

namespace nb {

const char* kind_name(Kind k) {
  switch (k) {
    case Kind::AllReduce: return "allreduce";
    case Kind::AllGather: return "allgather";
    case Kind::ReduceScatter: return "reducescatter";
    case Kind::Broadcast: return "broadcast";
    default: return "?";
  }
}

const char* dtype_name(DType t) {
  static const char* names[] = {"unsupported", "int8", "uint8", "int32", "uint32", "int64",
                                "uint64", "float16", "float32", "float64", "bfloat16",
                                "float8e4m3", "float8e5m2"};
  static_assert(sizeof(names) / sizeof(*names) == size_t(DType::Count), "dtype names");
  return names[size_t(t) < size_t(DType::Count) ? size_t(t) : 0];
}

const char* op_name(RedOp o) {
  static const char* names[] = {"sum", "prod", "max", "min", "avg", "premulsum", "unsupported"};
  static_assert(sizeof(names) / sizeof(*names) == size_t(RedOp::Count), "op names");
  return names[size_t(o) < size_t(RedOp::Count) ? size_t(o) : 6];
}

const char* algo_name(Algo a) {
  static const char* names[] = {"fallback", "ar_twoshot", "ar_nvls", "rs_pull", "ag_pull",
                                "bc_pull", "bc_scatter", "ar_staged", "rs_staged", "bc_chain",
                                "bc_nvls", "ag_nvls", "rs_nvls", "ag_push", "bc_ring", "rs_push", "ar_push", "ar_hybrid",
                                "ar_oneshot", "rs_hybrid", "ar_twoshot_ll", "rs_ll", "ag_ll", "bc_ll"};
  static_assert(sizeof(names) / sizeof(*names) == size_t(Algo::Count), "algo names");
  return names[size_t(a) < size_t(Algo::Count) ? size_t(a) : 0];
}

const char* reason_name(Reason r) {
  static const char* names[] = {
      "None", "NotGrouped", "UnsupportedType", "UnsupportedOp", "NullBuffer", "SizeOverflow",
      "BelowThreshold", "Misaligned", "BadSlot", "PartialOverlap", "BadRank", "GroupShape",
      "NotClique", "Mismatch", "Capturing", "FirstPass", "SetupFailed", "SubmitFailedEarly",
      "Poisoned", "AboveLimit", "AddressOverflow", "PolicyFallback", "MetadataQuery",
      "RuntimeUnsupported", "UnsupportedNccl", "Disabled", "FaultInjected", "DeviceTimeout"};
  static_assert(sizeof(names) / sizeof(*names) == size_t(Reason::Count), "reason names");
  return names[size_t(r) < size_t(Reason::Count) ? size_t(r) : 0];
}

size_t elem_size(DType t) {
  switch (t) {
    case DType::I8: case DType::U8: case DType::F8E4M3: case DType::F8E5M2: return 1;
    case DType::F16: case DType::BF16: return 2;
    case DType::I32: case DType::U32: case DType::F32: return 4;
    case DType::I64: case DType::U64: case DType::F64: return 8;
    default: return 0;
  }
}

bool reducible(DType t) {
  switch (t) {
    case DType::I8: case DType::U8: case DType::I32: case DType::U32: case DType::I64:
    case DType::U64: case DType::F16: case DType::F32: case DType::F64: case DType::BF16:
      return true;
    default:
      return false;  // fp8 reductions stay on NCCL
  }
}

bool is_float(DType t) {
  return t == DType::F16 || t == DType::F32 || t == DType::F64 || t == DType::BF16;
}

DType dtype_from_nccl(int t) {
  switch (t) {
    case nccl::Int8: return DType::I8;
    case nccl::Uint8: return DType::U8;
    case nccl::Int32: return DType::I32;
    case nccl::Uint32: return DType::U32;
    case nccl::Int64: return DType::I64;
    case nccl::Uint64: return DType::U64;
    case nccl::Float16: return DType::F16;
    case nccl::Float32: return DType::F32;
    case nccl::Float64: return DType::F64;
    case nccl::Bfloat16: return DType::BF16;
    case nccl::Float8e4m3: return DType::F8E4M3;
    case nccl::Float8e5m2: return DType::F8E5M2;
    default: return DType::Unsupported;
  }
}

int dtype_to_nccl(DType t) {
  switch (t) {
    case DType::I8: return nccl::Int8;
    case DType::U8: return nccl::Uint8;
    case DType::I32: return nccl::Int32;
    case DType::U32: return nccl::Uint32;
    case DType::I64: return nccl::Int64;
    case DType::U64: return nccl::Uint64;
    case DType::F16: return nccl::Float16;
    case DType::F32: return nccl::Float32;
    case DType::F64: return nccl::Float64;
    case DType::BF16: return nccl::Bfloat16;
    case DType::F8E4M3: return nccl::Float8e4m3;
    case DType::F8E5M2: return nccl::Float8e5m2;
    default: return -1;
  }
}

bool reduces(Kind k) { return k == Kind::AllReduce || k == Kind::ReduceScatter; }

size_t call_bytes(const CallDesc& c) { return c.count * elem_size(c.dtype); }

size_t send_extent(const CallDesc& c) {
  return c.kind == Kind::ReduceScatter ? size_t(c.nranks > 0 ? c.nranks : 1) * call_bytes(c)
                                       : call_bytes(c);
}

size_t recv_extent(const CallDesc& c) {
  return c.kind == Kind::AllGather ? size_t(c.nranks > 0 ? c.nranks : 1) * call_bytes(c)
                                   : call_bytes(c);
}

size_t logical_bytes(const CallDesc& c) {
  return (c.kind == Kind::AllGather || c.kind == Kind::ReduceScatter)
             ? size_t(c.nranks > 0 ? c.nranks : 1) * call_bytes(c)
             : call_bytes(c);
}

bool call_in_place(const CallDesc& c) {
  const size_t n = call_bytes(c);
  switch (c.kind) {
    case Kind::AllGather: return c.send == c.recv + size_t(c.rank) * n;
    case Kind::ReduceScatter: return c.recv == c.send + size_t(c.rank) * n;
    default: return c.send == c.recv;
  }
}

}  // namespace nb
