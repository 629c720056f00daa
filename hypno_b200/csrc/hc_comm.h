// Tensor-parallel communicator interface (see hc_comm.cu).
#pragma once
#include "hc_internal.h"

namespace hc {

struct Comm;

int comm_unique_id(uint8_t* out128);
int comm_init(Comm** out, const uint8_t* id128, int rank, int size, double timeout_s);
void comm_free(Comm* c);
int comm_allreduce_sum(Comm* c, float* buf, size_t count, cudaStream_t s);
int comm_allgather(Comm* c, const float* send, float* recv, size_t count, cudaStream_t s);
int comm_wait(Comm* c, cudaStream_t s, double timeout_s);

}  // namespace hc
