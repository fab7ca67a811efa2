// wb_decode.h -- fused decode step launcher.
#pragma once
#include "wave_b200.h"
#include "wb_internal.h"

namespace wb {

struct DecodeLaunch {
    WbSeqView sv;
    int32_t *len;
    int cap, n_slots;
    const float *x;
    const float *wrs_t, *brs, *wv_t, *bv, *wo_t, *bo, *hn;
    int n_seq, H, hd, E;
    float *y;
    uint32_t *dev_err;
};

// Scratch bytes the fused decode kernel needs for n_seq sequences; the
// ticket arrays inside must be zero before the first launch (the kernel
// leaves them zero).
size_t decode_scratch_bytes(int n_seq, int H, int hd, int E, int cap);
int launch_decode_fused(const DecodeLaunch &L, void *scratch, size_t scratch_bytes, cudaStream_t st,
                        std::string *msg);

}  // namespace wb
