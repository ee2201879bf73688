// Allocation-free staged AllReduce entry point.
//
// This entry point has no counterpart in the reference: it is an addition of
// this library.
//
// Who needs it: code that must not call cudaMalloc or any allocating library
// routine -- a caller running inside a CUDA-graph-capture-sensitive region, an
// allocator hook or a custom allocator of its own (where allocating would
// recurse), or a host that has already handed all device memory to its own
// pool. Such a caller passes its inputs and outputs and gets the staged
// AllReduce of N virtual ranks on the current device, with the staging
// scratch taken from a fixed device array that the library declares at file
// scope instead of from cudaMalloc.
//
// What it computes: for each rank r of `nranks` virtual ranks (all buffers on
// the current device), slice r of the message is staged -- every other
// rank's slice r is copied into the static scratch -- and one fold kernel
// sums the local slice and the staged ones in rank order (fp32 accumulation
// for 16-bit types) and writes the result into slice r of every rank's
// output: exactly the staged route's numerics (bit-identical to it).
//
// Limits and sharing:
//  * The scratch is a 32 MiB file-scope device array. With CUDA's default lazy
//    module loading only a GPU on which the entry point runs holds it, until
//    the process exits; with CUDA_MODULE_LOADING=EAGER the whole module loads
//    with the context, so every GPU the process (or an application that
//    preloads the interposer) initializes reserves the 32 MiB. A call is refused
//    (return value -2, message in `err`) when (nranks - 1) times the largest
//    slice exceeds 32 MiB.
//  * Every call shares that one array and it keeps the last call's contents;
//    nothing in it needs to start at zero (each slice is fully staged before
//    it is folded). Calls whose work overlaps on the GPU (different streams
//    without ordering) race on the array: order them on one stream.
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture.
//  * It calls no cudaMalloc, cudaFree or allocating library routine.
#pragma once

#include <cstddef>
#include <cstdint>

extern "C" {

enum {
  NB_NOALLOC_FLOAT16 = 6,   // ncclFloat16
  NB_NOALLOC_FLOAT32 = 7,   // ncclFloat32
  NB_NOALLOC_BFLOAT16 = 9,  // ncclBfloat16
};

// dtype: an ncclDataType_t value -- ncclFloat16 (6), ncclFloat32 (7) or
// ncclBfloat16 (9); the named constants below carry the same values.
// Returns 0 on success, -1 on bad arguments, -2 when the message is too large
// for the static scratch, or a CUDA error code; every non-zero return leaves
// a message in `err` (when errcap > 0).
int nb_staged_allreduce_noalloc(const void* const* sends, void* const* recvs, int nranks,
                                uint64_t count, int dtype, void* stream, char* err, size_t errcap);

// Capacity of the static scratch in bytes.
uint64_t nb_noalloc_scratch_bytes();
}
