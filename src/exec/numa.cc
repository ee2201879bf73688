// NUMA-local pinned host staging buffers for the PCIe host lane.
//
// Node: cudaDevAttrHostNumaId, the host node nearest the GPU as the driver
// reports it; where the driver has none, the numa_node file of the GPU's PCI
// function in sysfs.
//
// Placement: for the duration of one allocation the calling thread's memory
// policy binds to that node (set_mempolicy; the previous policy is restored
// afterwards). An anonymous mapping is created with MAP_POPULATE, so every
// page is faulted in now, by this thread, under that policy; the pages are
// then pinned for the GPU with cudaHostRegister (portable). The placement is
// checked page by page on an even sample of the buffer (get_mempolicy with
// MPOL_F_NODE | MPOL_F_ADDR answers the node a page lives on). Any failure
// frees what was made and falls back to cudaHostAlloc; the summary reports
// the target node, the node found and which method served.
//
// Parity: the reference's host bounce buffers (shim/nccl_collectives_shim.cu:
// 956-1078) are NUMA-local pinned memory placed with mbind and checked with
// move_pages.
#include <linux/mempolicy.h>
#include <sys/mman.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <array>
#include <cctype>
#include <fstream>
#include <string>
#include <vector>

#include "exec/executor.h"

namespace nb {

namespace {

// Bits in the node masks passed to the kernel (covers every node id a
// machine of this class can have; get_mempolicy refuses masks smaller than
// the kernel's node count).
constexpr unsigned long kMaskBits = 4096;
using NodeMask = std::array<unsigned long, kMaskBits / (8 * sizeof(unsigned long))>;

long sys_set_policy(int mode, const unsigned long* mask, unsigned long bits) {
  return syscall(SYS_set_mempolicy, mode, mask, bits);
}

// The node a page lives on, or -1.
int node_of_page(void* addr) {
  int node = -1;
  if (syscall(SYS_get_mempolicy, &node, nullptr, 0ul, addr, MPOL_F_NODE | MPOL_F_ADDR) != 0) return -1;
  return node;
}

// Binds this thread's allocations to one node while alive; restores the
// thread's previous policy on destruction.
class ThreadNodeBinding {
 public:
  explicit ThreadNodeBinding(int node) {
    NodeMask old{};
    if (syscall(SYS_get_mempolicy, &old_mode_, old.data(), kMaskBits, nullptr, 0ul) != 0) return;
    old_mask_ = old;
    saved_ = true;
    NodeMask want{};
    want[size_t(node) / (8 * sizeof(unsigned long))] |= 1ul << (size_t(node) % (8 * sizeof(unsigned long)));
    bound_ = sys_set_policy(MPOL_BIND, want.data(), kMaskBits) == 0;
  }
  ~ThreadNodeBinding() {
    if (!bound_) return;
    if (old_mode_ == MPOL_DEFAULT) sys_set_policy(MPOL_DEFAULT, nullptr, 0);
    else sys_set_policy(old_mode_, old_mask_.data(), kMaskBits);
  }
  bool bound() const { return saved_ && bound_; }
  ThreadNodeBinding(const ThreadNodeBinding&) = delete;
  ThreadNodeBinding& operator=(const ThreadNodeBinding&) = delete;

 private:
  int old_mode_ = MPOL_DEFAULT;
  NodeMask old_mask_{};
  bool saved_ = false, bound_ = false;
};

// The node every sampled page of [p, p + len) lives on, or -1 when they
// differ or cannot be read: pages at each eighth of the buffer and its last.
int placement_of(void* p, size_t len, size_t page) {
  if (!p || !len || !page) return -1;
  std::vector<size_t> offsets;
  for (int k = 0; k < 8; ++k) offsets.push_back(len / 8 * size_t(k) / page * page);
  offsets.push_back((len - 1) / page * page);
  int node = -2;
  for (size_t off : offsets) {
    const int here = node_of_page(static_cast<char*>(p) + off);
    if (here < 0 || (node != -2 && here != node)) return -1;
    node = here;
  }
  return node;
}

int sysfs_numa_node(int dev) {
  char bus[64] = {};
  if (cudaDeviceGetPCIBusId(bus, sizeof bus, dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  std::string id(bus);
  std::transform(id.begin(), id.end(), id.begin(), [](unsigned char c) { return char(std::tolower(c)); });
  const bool plain = !id.empty() && std::all_of(id.begin(), id.end(), [](unsigned char c) {
    return std::isxdigit(c) || c == ':' || c == '.';
  });
  if (!plain) return -1;
  std::ifstream in("/sys/bus/pci/devices/" + id + "/numa_node");
  int node = -1;
  return (in >> node) ? node : -1;
}

}  // namespace

int gpu_numa_node(int dev) {
  int node = -1;
  if (cudaDeviceGetAttribute(&node, cudaDevAttrHostNumaId, dev) == cudaSuccess && node >= 0) return node;
  cudaGetLastError();
  return sysfs_numa_node(dev);
}

void* alloc_pinned_near(int dev, size_t bytes, size_t* mapped, int* target_out, int* placed_out,
                        const char** method) {
  *mapped = 0;
  *placed_out = -1;
  const int target = gpu_numa_node(dev);
  *target_out = target;
  const long sz = sysconf(_SC_PAGESIZE);
  const size_t page = sz > 0 ? size_t(sz) : 0;
  const bool placeable = target >= 0 && size_t(target) < kMaskBits && page && bytes > 0 &&
                         bytes <= ~size_t(0) - page;
  if (placeable) {
    const size_t len = (bytes + page - 1) / page * page;
    void* p = MAP_FAILED;
    {
      ThreadNodeBinding bind(target);
      if (bind.bound())
        p = mmap(nullptr, len, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS | MAP_POPULATE, -1, 0);
    }
    if (p != MAP_FAILED) {
      const int placed = placement_of(p, len, page);
      *placed_out = placed;
      if (placed == target && cudaHostRegister(p, len, cudaHostRegisterPortable) == cudaSuccess) {
        *mapped = len;
        *method = "bound";
        return p;
      }
      cudaGetLastError();
      munmap(p, len);
    }
  }
  void* p = nullptr;
  if (cudaHostAlloc(&p, bytes, cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  *placed_out = page ? placement_of(p, bytes, page) : -1;
  *method = "fallback";
  return p;
}

bool free_pinned(void* p, size_t bytes, size_t mapped) {
  if (!p) return true;
  bool ok = true;
  if (mapped) {
    ok = cudaHostUnregister(p) == cudaSuccess;
    if (!ok) cudaGetLastError();
    return ok && munmap(p, mapped) == 0;
  }
  (void)bytes;
  ok = cudaFreeHost(p) == cudaSuccess;
  if (!ok) cudaGetLastError();
  return ok;
}

}  // namespace nb
