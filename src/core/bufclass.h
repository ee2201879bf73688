// Classification of a caller's buffer from the facts the CUDA driver reports
// about it, as a pure function (no CUDA here; the executor gathers the facts).
//
// A collective may read or write a caller's buffer from every GPU of the
// clique, so the buffer must be one allocation that peers can reach. Two
// kinds qualify:
//   Ordinary  cudaMalloc memory (legacy-IPC capable), reached through peer
//             access; the access query has no per-device mapping for it
//             (INVALID_VALUE) or reports no flags or read-write.
//   Mapped    VMM memory (cuMemCreate/cuMemMap, e.g. ncclMemAlloc), not
//             legacy-IPC capable, mapped read-write for every clique device.
// Anything else is refused, with the first failing rule of the table named:
// a pointer the driver does not know, host or managed memory, the wrong
// device, a range that leaves its allocation, memory from a stream-ordered
// pool (cudaMallocAsync memory is not made peer-accessible by
// cudaDeviceEnablePeerAccess), or facts that fit neither kind. The facts are
// taken at the first and at the last byte, since a VMM range can join
// separately mapped pieces.
//
// Parity: the reference's supported_buffer (shim/nccl_collectives_shim.cu:
// 1635-1705) classifies a pair's buffers by the same attributes.
#pragma once

#include <cstddef>
#include <cstdint>

#include "core/types.h"

namespace nb {

// Outcome of the per-device access query (cuMemGetAccess) at one byte.
enum class Access : uint8_t { NoMapping, NoFlags, ReadWrite, OtherFlags, QueryFailed };

struct PointerFacts {
  bool known = false;          // the attribute query succeeded
  bool device_memory = false;  // CU_MEMORYTYPE_DEVICE
  int device = -1;             // ordinal of the owning device
  uint64_t range_start = 0;    // the allocation (address range) holding this byte
  uint64_t range_size = 0;
  uint64_t mapping_start = 0;  // the physical mapping holding it (0 when not reported)
  uint64_t mapping_size = 0;
  bool from_pool = false;      // stream-ordered allocator memory
  int legacy_ipc = -1;         // 1 capable, 0 not, -1 unknown
  int ndev = 0;
  Access access[kMaxRanks] = {};  // per clique device
};

enum class BufferClass : uint8_t { Refused, Ordinary, Mapped };

struct BufferVerdict {
  BufferClass cls = BufferClass::Refused;
  const char* rule = "";  // the rule that decided (the failing one when refused)
};

// `first` and `last` describe bytes addr and addr + bytes - 1.
BufferVerdict classify_buffer(const PointerFacts& first, const PointerFacts& last, uint64_t addr,
                              uint64_t bytes, int expected_device);

}  // namespace nb
