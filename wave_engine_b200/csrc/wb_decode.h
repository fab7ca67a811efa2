// wb_decode.h -- decode step launchers.
#pragma once
#include "wave_b200.h"
#include "wb_internal.h"

namespace wb {

struct DecodeLaunch {
    WbSeqView sv;
    int32_t *len;
    int cap, n_slots;
    const float *x;
    const float *wrs_h, *brs, *wv_t, *bv, *wo_t, *bo, *hn;  // wrs_h: [H][E][2]
    int n_seq, H, hd, E;
    int sm_count;
    uint32_t *dev_err;
    // launch the attention grid as a programmatic dependent of the previous
    // kernel in the stream; only when that kernel, if it is this library's
    // decode out_proj, served another layer or cache (see tc_kv_decode)
    bool chain;
};

// Scratch bytes the decode attention kernel needs for n_seq sequences; the
// ticket arrays inside must be zero before the first launch (the kernel
// leaves them zero).
size_t decode_scratch_bytes(int n_seq, int H, int hd, int E, int cap);
// Byte range of the ticket counters inside that scratch.
void decode_scratch_tickets(int n_seq, int H, int hd, int E, int cap, size_t *offset, size_t *bytes);
// Attention part of one decode step (one launch): writes the merged,
// normalised head outputs o [n_seq][E] (inside scratch, returned in
// *o_out) and appends the new position to every slot; out_proj and the
// length update follow in later launches.
int launch_decode_attn(const DecodeLaunch &L, void *scratch, size_t scratch_bytes, float **o_out,
                       cudaStream_t st, std::string *msg);

// y = o W_o^T + b for the step's n rows (wo_t input-major), then
// len[slot[i]] += 1 for every row whose length is below cap (and, with a
// page table, whose next position's page is mapped).  Launched as a
// programmatic dependent of the attention grid.
int launch_decode_out(const float *o, const float *wo_t, const float *bo, float *y, int n, int E, int cap,
                      int32_t *len, const int32_t *slot, int n_slots, cudaStream_t st, std::string *msg,
                      const int32_t *pages = nullptr, int max_pages = 0);

}  // namespace wb
