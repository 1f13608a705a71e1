// model.h -- device state of a decode model (one tensor-parallel rank), shared by engine.cu and the
// exchanges of comm.cu.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <vector>

#include "../../include/pox_cuda.h"
#include "api_internal.h"
#include "comm.cuh"

namespace pox {

constexpr int kPage = 16;       // tokens per KV page (paged_cache.rs DEFAULT_BLOCK_SIZE)
constexpr int kSplitTok = 64;   // context tokens per attention CTA (4 pages)
constexpr int kArgmaxParts = 64;  // max blocks per row of the argmax's first pass

// One layer's projections as the persistent decode kernel reads them (persist.cu): the INT4 tile
// blobs of qkv, o, gate_up and down, and the two f16 norm weights.
struct PLayer {
    const uint8_t* w[4];
    const uint16_t* attn_norm;
    const uint16_t* mlp_norm;
};

struct LayerW {
    pox_tensor* qkv = nullptr;
    pox_tensor* o = nullptr;
    pox_tensor* gu = nullptr;
    pox_tensor* down = nullptr;
    uint16_t* attn_norm = nullptr;
    uint16_t* mlp_norm = nullptr;
};

}  // namespace pox

// Sizes are this rank's shard: nq, nkv, I and V are the whole model's divided by tp.
struct pox_model {
    pox_cuda_ctx* ctx = nullptr;
    pox_llama_config cfg{};
    int H = 0, I = 0, V = 0, L = 0, nq = 0, nkv = 0, hd = 0, G = 0, qkv_rows = 0;
    int V_full = 0, vocab_off = 0;  // embedding rows; first vocab row of this rank's lm_head slice
    uint32_t max_batch = 0, kv_blocks = 0, max_blocks_per_seq = 0;
    uint16_t* embed = nullptr;
    uint16_t* final_norm = nullptr;
    pox_tensor* lm_head = nullptr;
    std::vector<pox::LayerW> layers;
    __half* kc = nullptr;  // [kv_blocks][L][nkv][16][hd]
    __half* vc = nullptr;
    float* x = nullptr;       // [B][H] residual stream
    float* qkv = nullptr;     // [B][qkv_rows]
    float* att = nullptr;     // [B][nq * hd]
    float* gu = nullptr;      // [B][2 I]
    float* logits = nullptr;  // [B][V]
    float* apart = nullptr;   // [B][nkv][max_splits][G][hd + 2]
    float2* rope = nullptr;   // [max_blocks_per_seq * 16][hd / 2]: (cos, sin) of RoPE pair i at position p
    float2* amax = nullptr;   // [B][kArgmaxParts] first-pass argmax pairs
    uint32_t* tok = nullptr;  // [B]
    uint32_t* pos = nullptr;  // [B]
    uint32_t* next = nullptr; // [B]
    int32_t* btab = nullptr;  // [B][max_blocks_per_seq]
    uint32_t* sel = nullptr;  // [B] prefill: rows whose logits are returned
    float* xsel = nullptr;    // [B][H] prefill: those rows of x
    int max_splits = 0;
    pox::TpComm comm;
    // persistent decode kernel (persist.cu): per-layer tile pointers, (sequence, kv head) combine
    // tickets [max_batch][nkv], grid-barrier words [4]; persist = 1 runs qualifying decode steps on it
    pox::PLayer* players = nullptr;
    uint32_t* ptickets = nullptr;
    unsigned* pbar = nullptr;
    float* pssq = nullptr;       // [H / 16][2][4] sums of squares of the residual rows
    std::vector<uint8_t> pready;  // layer l's entry of players is current
    int persist = 0;
};
