// 2-D exact SIMT engine (exact2d.cu): small IVF batches, every distance
// exact in the reference order, three launches over (slice, frame) grids.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "kernels.h"

namespace vfr {

struct Exact2dArgs {
    ExactArgs e;   // index arrays, frames, outputs, mode (frame_list unused)
    int slices;    // coarse CTAs per frame (32 centroids each)
    int parts;     // fine CTAs per frame (64 scan positions each)
    int probes;    // min(nprobe, nlist)
    unsigned long long *coarse_keys;  // [frames][slices][probes]
    unsigned long long *fine_keys;    // [frames][parts][8]
    int32_t *probe_list;              // [frames][probes]
    uint32_t *probe_base;             // [frames][probes + 1]
};

// Byte offsets of the engine's scratch for `frames` frames; max_probed is the
// largest number of rows a frame's probed lists can hold (the sum of the
// nprobe largest lists).
struct Exact2dLayout {
    int slices, parts, probes;
    size_t coarse_keys, fine_keys, probe_list, probe_base, total;
};
Exact2dLayout exact2d_layout(size_t frames, int nlist, int nprobe, int64_t max_probed);

// Widest rows the engine takes (its coarse stage stages rows in shared memory).
int exact2d_max_width();

// Enqueues the three launches on `s` (workspace laid out by `l`).
void launch_exact2d(const ExactArgs &e, void *workspace, const Exact2dLayout &l, long long frames, cudaStream_t s);

}  // namespace vfr
