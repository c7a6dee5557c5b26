// gpb2_comm.h -- the collectives the level-sharded operations use (gpb2_comm.cu, NCCL).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/graphgp_b200.h"

namespace gpb2 {

int comm_rank(const gpb2_comm* c);
int comm_size(const gpb2_comm* c);
int64_t comm_min_shard(const gpb2_comm* c);
// In place: buf[lo + r*count : lo + (r+1)*count] of every rank r -> buf[lo : lo + size*count].
int comm_all_gather(gpb2_comm* c, void* buf, int64_t lo, int64_t count, bool f64, cudaStream_t s);
// In place: the sum over ranks of buf[lo : lo + size*count] -> this rank's part
// buf[lo + rank*count : lo + (rank+1)*count].
int comm_reduce_scatter(gpb2_comm* c, void* buf, int64_t lo, int64_t count, bool f64,
                        cudaStream_t s);
// In place sum over ranks of buf[0 : count].
int comm_all_reduce(gpb2_comm* c, void* buf, int64_t count, bool f64, cudaStream_t s);

}  // namespace gpb2
