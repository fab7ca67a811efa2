// wb_tc.cu -- WB_PATH_TENSOR sequencing (placeholder until the tcgen05
// kernels land: every entry reports WB_ENOTSUP).
#include "wb_tc.h"

namespace wb {

int tc_layer_upload(TcLayerWeights *t, const wb_attn_weights_desc *w, const float *, std::string *) {
    t->E = w->n_embd;
    t->H = w->n_head;
    t->hd = w->n_embd / w->n_head;
    t->C = w->content_dim;
    return WB_OK;
}
void tc_layer_free(TcLayerWeights *) {}

int tc_attn_forward(const TcLayerWeights &, const float *, int, int, bool, float *, float *, Workspace *,
                    uint32_t *, int, cudaStream_t, std::string *msg) {
    *msg = "WB_PATH_TENSOR not built yet";
    return WB_ENOTSUP;
}
int tc_kv_prefill(const TcLayerWeights &, const WbSeqView &, const float *, int, int, float *, Workspace *,
                  uint32_t *, int, cudaStream_t, std::string *msg) {
    *msg = "WB_PATH_TENSOR not built yet";
    return WB_ENOTSUP;
}
int tc_kv_decode(const TcLayerWeights &, const WbSeqView &, const int32_t *, int, const float *, int, float *,
                 Workspace *, uint32_t *, int, cudaStream_t, std::string *msg) {
    *msg = "WB_PATH_TENSOR not built yet";
    return WB_ENOTSUP;
}

}  // namespace wb
