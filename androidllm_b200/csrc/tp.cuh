// Internal interface of the run-time loaded NCCL (tp.cu).  Every function
// returns 0 on success, else nonzero with a message in *err.
#pragma once
#include <cuda_runtime.h>

#include <string>

namespace alm {

constexpr int kTpIdBytes = 128;   // NCCL unique id

int tp_unique_id(unsigned char* out, std::string* err);
int tp_comm_init(int rank, int world, const unsigned char* id, void** comm, std::string* err);
void tp_comm_destroy(void* comm);
int tp_allreduce_sum_f32(void* comm, float* buf, size_t n, cudaStream_t st, std::string* err);
int tp_allgather(void* comm, const void* send, void* recv, size_t bytes_per_rank, cudaStream_t st,
                 std::string* err);

}  // namespace alm
