// NUMA-local pinned host staging buffers for the PCIe host lane.
//
// The GPU's NUMA node comes from cudaDevAttrNumaId when the runtime has it,
// else from /sys/bus/pci/devices/<bdf>/numa_node. The buffer is an anonymous
// mapping bound to that node (mbind MPOL_BIND, STRICT|MOVE), first-touched,
// verified with move_pages on up to 16 sampled pages, then registered with
// cudaHostRegister(Portable). Any failure falls back to cudaHostAlloc.
//
// Parity: staging_numa_node / staging_placement / allocate_bounce /
// free_bounce of the reference (shim/nccl_collectives_shim.cu:956-1078).
#include <linux/mempolicy.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <cctype>
#include <cstdio>
#include <vector>

#include "exec/executor.h"

namespace nb {

int gpu_numa_node(int dev) {
  int node = -1;
  if (cudaDeviceGetAttribute(&node, cudaDevAttrNumaId, dev) == cudaSuccess && node >= 0) return node;
  cudaGetLastError();
  char pci[32] = {};
  if (cudaDeviceGetPCIBusId(pci, sizeof(pci), dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  for (char* c = pci; *c; ++c) {
    const unsigned char v = static_cast<unsigned char>(*c);
    if (!std::isxdigit(v) && *c != ':' && *c != '.') return -1;
    *c = static_cast<char>(std::tolower(v));
  }
  char path[96];
  std::snprintf(path, sizeof(path), "/sys/bus/pci/devices/%s/numa_node", pci);
  FILE* f = std::fopen(path, "r");
  if (!f) return -1;
  int placed = -1;
  const bool parsed = std::fscanf(f, "%d", &placed) == 1;
  std::fclose(f);
  return parsed ? placed : -1;
}

static int sampled_placement(void* p, size_t n, size_t page) {
  if (!n || !page) return -1;
  const size_t pages = 1 + (n - 1) / page;
  const size_t count = pages < 16 ? pages : 16;
  void* addresses[16];
  int status[16];
  for (size_t i = 0; i < count; ++i) {
    const size_t index = count == 1 ? 0 : (pages - 1) * i / (count - 1);
    addresses[i] = static_cast<char*>(p) + index * page;
    status[i] = -1;
  }
  if (syscall(SYS_move_pages, 0, count, addresses, nullptr, status, 0) != 0) return -1;
  for (size_t i = 0; i < count; ++i)
    if (status[i] < 0 || status[i] != status[0]) return -1;
  return status[0];
}

void* alloc_pinned_near(int dev, size_t bytes, size_t* mapped, int* target_out, int* placed_out,
                        const char** method) {
  *mapped = 0;
  const int target = gpu_numa_node(dev);
  *target_out = target;
  *placed_out = -1;
  const long page_size = sysconf(_SC_PAGESIZE);
  const size_t page = page_size > 0 ? size_t(page_size) : 0;
  if (target >= 0 && target < 4096 && page && bytes <= SIZE_MAX - (page - 1)) {
    const size_t rounded = ((bytes + page - 1) / page) * page;
    void* p = mmap(nullptr, rounded, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
    if (p != MAP_FAILED) {
      constexpr size_t bits = sizeof(unsigned long) * 8;
      std::vector<unsigned long> mask(size_t(target) / bits + 2, 0);
      mask[size_t(target) / bits] |= 1UL << (size_t(target) % bits);
      bool ok = syscall(SYS_mbind, p, rounded, MPOL_BIND, mask.data(),
                        static_cast<unsigned long>(mask.size() * bits), MPOL_MF_STRICT | MPOL_MF_MOVE) == 0;
      if (ok) {
        for (size_t off = 0; off < rounded; off += page) static_cast<volatile unsigned char*>(p)[off] = 0;
        const int placed = sampled_placement(p, rounded, page);
        *placed_out = placed;
        ok = placed == target;
      }
      if (ok && cudaHostRegister(p, rounded, cudaHostRegisterPortable) == cudaSuccess) {
        *mapped = rounded;
        *method = "mbind";
        return p;
      }
      cudaGetLastError();
      munmap(p, rounded);
    }
  }
  void* p = nullptr;
  if (cudaHostAlloc(&p, bytes, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  *placed_out = page ? sampled_placement(p, bytes, page) : -1;
  *method = "fallback";
  return p;
}

bool free_pinned(void* p, size_t bytes, size_t mapped) {
  if (!p) return true;
  if (mapped) {
    if (cudaHostUnregister(p) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    return munmap(p, mapped) == 0;
  }
  (void)bytes;
  if (cudaFreeHost(p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return true;
}

}  // namespace nb
