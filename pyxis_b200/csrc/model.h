// model.h -- the decode model handle behind include/pyxis_decode.h, shared by decode.cu (one
// sequence) and decode_batch.cu (many sequences).
#pragma once

#include <vector>

#include "../../include/pyxis_comm.h"
#include "../../include/pyxis_decode.h"
#include "ctx.h"
#include "kernels.h"

namespace pyxis {
struct BatchState;
void free_batch_state(BatchState *b);

// The fused decode attention (decode.cu) over n_seq sequences at the same position: sequence z
// reads its q|k|v row at qkv + z * qkv_stride, its KV cache (this layer) at kc/vc + z * cache_stride,
// and writes its attention output at out + z * out_stride.  part / tickets hold n_seq * n_kv *
// splits partials and n_seq * n_kv tickets (zero before the first launch; left zero).
cudaError_t launch_attention_step(const pyxis_model_config &c, int splits, int n_seq, const float *qkv,
                                  size_t qkv_stride, const float *q_norm, const float *k_norm, const float *rope_cos,
                                  const float *rope_sin, const int *d_pos, float *kc, float *vc, size_t cache_stride,
                                  float *part, unsigned *tickets, float *out, size_t out_stride, cudaStream_t st);
}  // namespace pyxis

struct pyxis_cuda_model {
    pyxis_cuda_ctx *ctx = nullptr;
    pyxis_model_config cfg{};
    int q_dim = 0, kv_dim = 0;
    struct Layer {
        const pyxis_cuda_weights *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr;
        float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    };
    std::vector<Layer> layers;
    uint16_t *emb = nullptr;
    const pyxis_cuda_weights *lm_head = nullptr;
    float *final_norm = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    float *kcache = nullptr, *vcache = nullptr;
    float *x2 = nullptr;                      // the residual stream alternates between x and x2
    float *part = nullptr;                    // attention split partials [n_kv][splits][G][hd + 2]
    unsigned *tickets = nullptr;              // [n_kv], zero between launches
    int attn_splits = 1;
    float *x = nullptr, *h = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *tmp = nullptr, *gu = nullptr,
          *act = nullptr, *logits = nullptr;
    int *d_pos = nullptr, *d_token = nullptr, *d_step = nullptr, *d_out = nullptr;
    cudaGraphExec_t exec = nullptr;
    std::vector<void *> allocs;
    pyxis::BatchState *batch = nullptr;  // buffers of pyxis_cuda_model_generate_batch (decode_batch.cu)
    // vocab-parallel head of pyxis_cuda_model_generate_batch (pyxis_cuda_model_set_vocab_parallel)
    pyxis_cuda_comm *vp_comm = nullptr;
    const pyxis_cuda_weights *vp_shard = nullptr;
    size_t vp_lo = 0, vp_rows = 0;
};
