// Pushing one device buffer into up to 7 peer buffers (this rank's slot in
// the other ranks' gather buffers, mapped through CUDA IPC).
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

namespace mb {

constexpr int kMaxPushPeers = 7;

// Copies `bytes` (a multiple of 4) from `src` to every `peers[d]`, d <
// num_peers, with one kernel on `s`: each thread loads 16 bytes once and
// stores them to every peer, so all peers' NVLink ports carry data at once
// (copy-engine copies issued one after another on a stream run one peer at
// a time). Ends with a system-scope fence; it never waits on another GPU.
void push_to_peers(const void* src, void* const* peers, int num_peers, size_t bytes,
                   cudaStream_t s);

}  // namespace mb
