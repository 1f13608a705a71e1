// comm.cuh -- the exchanges of tensor-parallel decode: the sum of the row-split projections'
// partial outputs (after o_proj and after down_proj, one per layer each) and the gather of each
// rank's best (logit, token) pair for the greedy pick over the whole vocabulary.
//
// Two implementations behind one interface:
//  * NCCL: ncclAllReduce in place on the residual stream (rank 0's partial carries the residual)
//    and ncclAllGather of the (logit, token) pairs.
//  * Peer: one-shot kernels over CUDA IPC mappings of every rank's exchange buffer. A rank's GEMV
//    writes its partial into its own buffer; the exchange kernel announces arrival to every rank
//    (a release store of the exchange's epoch into each rank's flag array), waits until every rank
//    announced the same epoch (acquire loads, bounded by kWaitCycles, then an error flag), and
//    sums all ranks' partials element by element in rank order, so every rank computes bit-identical
//    results. Epoch = decode steps completed (a device counter) x exchanges per step + exchange
//    index + 1, so the kernels capture into CUDA graphs unchanged.
//    Buffer reuse: allreduce k uses data slot k % 2 and the pair gather its own region. A rank
//    rewrites a slot only after completing a later exchange, which every rank joined only after
//    finishing its reads of that slot, so two slots suffice.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace pox {

constexpr int kMaxTP = 8;
constexpr int kErrWaitPeer = 8;  // bit of the kernel error flag: a peer never arrived

struct PeerView {                          // kernel parameter of the peer exchanges
    float* slot[kMaxTP][3];                // every rank's data slots 0, 1 and pair region 2 (mapped here)
    unsigned long long* flags[kMaxTP];     // every rank's arrival flags [kMaxTP] (index = source rank)
    unsigned long long* step;              // decode steps completed (this rank's device counter)
    int* err;                              // context error flag (host-mapped)
    int* abort;                            // sticky: a wait of this rank expired (local device word)
    int rank, tp;
};

struct TpComm {
    int rank = 0, tp = 1, mode = 0;
    void* nccl = nullptr;                  // ncclComm_t
    char* buf = nullptr;                   // this rank's exchange buffer (IPC-exported)
    size_t slot_bytes = 0, pair_bytes = 0;
    void* mapped[kMaxTP] = {};             // opened IPC mappings of the other ranks' buffers
    bool peer_ready = false;
    unsigned long long* step = nullptr;    // device counter of completed decode steps
    float2* pairs = nullptr;               // [max_batch] this rank's best (logit, token) per row
    float2* gathered = nullptr;            // [tp][max_batch] (NCCL gather target)
    PeerView view{};
};

// Exchange buffer layout: [flags: kMaxTP x u64 at 0, this rank's abort word at 128, padded to
// 256 B] [slot 0] [slot 1] [pair region].
int comm_alloc(TpComm& c, int rank, int tp, size_t max_batch, size_t hidden, int* err_dev);
void comm_free(TpComm& c);
int comm_init_nccl(TpComm& c, const uint8_t id[128]);
int comm_ipc_handle(TpComm& c, uint8_t handle[64]);
int comm_open_peers(TpComm& c, const uint8_t* handles);
// Where exchange `call` (0 .. 2 layers - 1) expects this rank's partial of n floats: the residual
// stream itself for NCCL (summed in place), the call's data slot for the peer exchange.
float* comm_partial(TpComm& c, int call, float* x);
// Clears the abort word (start of a host-driven decode call).
int comm_reset(TpComm& c, cudaStream_t st);
// x = sum over ranks of the partials (in place for NCCL); calls_per_step = 2 layers + 1.
int comm_allreduce(TpComm& c, int call, int calls_per_step, float* x, size_t n, cudaStream_t st);
// next[b] = the first maximum over the ranks' pairs (c.pairs of every rank, vocab slices in rank
// order); advances the step counter.
int comm_pick(TpComm& c, int call, int calls_per_step, int B, uint32_t* next, cudaStream_t st);

}  // namespace pox
