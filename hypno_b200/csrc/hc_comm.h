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
// Every rank's `bytes` host bytes gathered in rank order into recv (blocking).
int comm_allgather_host(Comm* c, const void* send, void* recv, size_t bytes);

// One-shot peer all-reduce fused with the residual add and the next RMSNorm
// (hc_peer_ar.cu), for decode-sized row-parallel outputs.
struct PeerAr;
int peer_ar_init(Comm* c, int rank, int size, size_t rows_cap, size_t H, PeerAr** out);
void peer_ar_free(PeerAr* a, int rank, int size);
// This rank's [rows_cap][H] partial buffer of slot 0 (o_proj) or 1
// (down_proj); the two slots must alternate from call to call.
float* peer_ar_partial(PeerAr* a, int slot);
bool peer_ar_fits(const PeerAr* a, size_t rows, size_t H);
// hidden[r] += sum over ranks of partial[r] of the slot (rank order); then,
// when w is not null, xn[r] = RMSNorm(hidden[r]) * w and its fp16 copy in
// GEMM K order.  slabs (may be null): this rank's product as `splits`
// split-K slabs of [rows][H] (local memory), added in slab order into the
// slot's partial first; null: the partial already holds the product.
int peer_ar_residual_norm(PeerAr* a, int slot, int rank, int size, size_t rows, const float* slabs, int splits,
                          float* hidden, size_t ldh, const float* w, float eps, float* xn, size_t ldxn, __half* xn16,
                          int* err, cudaStream_t s);

}  // namespace hc
