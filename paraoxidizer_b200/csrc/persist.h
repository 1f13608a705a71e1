// persist.h -- the persistent decode kernel (persist.cu): arguments and host entry points.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "model.h"

namespace pox {

constexpr int kPMaxB = 4;  // batch rows of one persistent launch

struct PArgs {
    const PLayer* layers;
    int L;
    int nT[4], nkb[4];  // row tiles and 128-k blocks of qkv, o, gate_up, down (the same in every layer)
    float* x;           // [B][H] residual stream
    float* qkv;         // [B][qkv_rows]
    float* att;         // [B][nq * 128]
    float* gu;          // [B][2 I]
    float* apart;       // [B][nkv][max_splits][G][130] attention split partials
    const uint32_t* pos;
    const int32_t* btab;
    __half* kc;
    __half* vc;
    const float2* rope;
    uint32_t* tickets;  // [B][nkv], zero between launches
    float* ssq;         // [H / 16][2][4] sums of squares of the residual rows each o / down row tile wrote
    unsigned* bar;      // [4]: barrier arrivals, unused, abort word, exits (zero between launches)
    int* err;
    int B, H, I, nq, nkv, G, qkv_rows, mbps, kv_blocks, max_splits;
    float eps;
    int S;                          // ring stages per warp
    int off_x, off_xm, off_red, off_lys, cs, nxbs;  // shared-memory plan
};

// Whether a decode step of `batch` rows can run as one persistent launch: one GPU, batch <= 4,
// head_dim 128 with 4..8 query heads per kv head, every projection INT4 in the tiled layout with
// group size 128 and no outliers, and the shared-memory plan fits.
bool persist_supported(const pox_model* m, int batch);
// Records layer l's tile pointers for the kernel (after its tensors are set). Synchronous.
int persist_set_layer(pox_model* m, int l);
// Launches the layers of one decode step (embedding done, lm_head to follow) on `st`.
int persist_launch(pox_model* m, int batch, cudaStream_t st);

}  // namespace pox
