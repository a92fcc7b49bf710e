// peer.h — tensor parallelism over NVLink peer memory (peer.cu).
#pragma once
#include <cuda_runtime.h>
#include <cstdint>

namespace lx2v {

constexpr int LX2V_MAX_PEERS = 8;

// flags[r]: rank r's flag array (world u32 slots), as this rank's device
// addresses it (its own, or a CUDA IPC mapping of a peer's).
struct PeerFlags {
    unsigned *flags[LX2V_MAX_PEERS];
};

// The step after a row-split linear, on rows [row0, row1) of an M x dim
// output: h[r] += gate * sum_p parts[p][r] (no add when n_parts == 0), then
// norm(h[r]) into outs[p][r] for every p (bf16 or f32). h is f32.
struct TpNormArgs {
    const void *parts[LX2V_MAX_PEERS];
    int parts_f32, n_parts;
    void *h;
    int64_t row0, row1;
    int dim;
    const void *gmods; int gmods_f32; int gate;   // gate < 0: h += sum
    int kind;                                      // 0 affine (w, b), 1 modulated (nmods rows scale, shift)
    const void *w; int w_f32;
    const void *b; int b_f32;
    const void *nmods; int nmods_f32; int scale, shift;
    float eps;
    void *outs[LX2V_MAX_PEERS];
    int out_f32, n_outs;
};

// Row sums of squares of columns [col_off, col_off + width) of src, written
// at outs[p][slot + r] for every rank p (the slot of this rank).
struct PeerRowSums {
    const void *src; int src_f32;
    int64_t rows, stride, col_off;
    int width;
    float *outs[LX2V_MAX_PEERS];
    int n_outs;
    int64_t slot;
};
cudaError_t row_sumsq_peers_launch(const PeerRowSums &a, cudaStream_t st);

cudaError_t peer_barrier_launch(const PeerFlags &f, int world, int rank, unsigned epoch, int *err, uint64_t limit_ns,
                                cudaStream_t st);
bool tp_reduce_norm_supported(int dim);  // dim a multiple of 8, at most 8192
cudaError_t tp_reduce_norm_launch(const TpNormArgs &a, cudaStream_t st);

}  // namespace lx2v
