// The row-shard table of the peer blend: where each shard's fp32 rows live
// (this process's mapping: a CUDA IPC mapping, another device of this
// process, or this device) and the global label bounds of the shards.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace vfr {

constexpr int kMaxPeerShards = 64;

struct PeerTable {
    int shards;
    int d;
    const float *rows[kMaxPeerShards];         // [rows of shard][d]
    const int32_t *row_of_id[kMaxPeerShards];  // null: identity (labels are storage rows)
    int64_t bounds[kMaxPeerShards + 1];        // global label bounds of the shards
};

// The reference's weights and blend of `frames` frames from their merged
// top-8 (dist, global labels [frames][8]), each winner's row read from the
// shard that owns it with plain loads (crates/vocal-cpu/src/retrieval.rs:65-81).
void launch_blend_peer(const PeerTable &t, const float *queries, float *out, const float *dist,
                       const int64_t *labels, long long frames, const float *index_rate, cudaStream_t stream);

}  // namespace vfr
