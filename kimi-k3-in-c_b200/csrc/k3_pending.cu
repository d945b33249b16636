// k3_pending.cu -- entry points declared in the headers whose device bodies are not
// built yet. Each records K3D_EUNSUPPORTED and returns.
#include "k3_common.cuh"

using namespace k3;

extern "C" {

long k3_expert_drops = 0;

int k3_is_mla(const K3Cfg *c, int layer)
{
    for (int i = 0; i < c->n_full_attn; i++)
        if (c->full_attn[i] == layer + 1) return 1;
    return 0;
}
int k3_is_kda(const K3Cfg *c, int layer) { return !k3_is_mla(c, layer); }
int k3_is_dense(const K3Cfg *c, int layer) { return layer < c->first_dense; }

#define PENDING(name) fail(K3D_EUNSUPPORTED, "%s is not built yet", name)

size_t k3_mla_scratch_cached(const K3Cfg *c, int T, int cap, int cached_mode) { PENDING("k3_mla_scratch_cached"); return 0; }
size_t k3_mla_scratch(const K3Cfg *c, int T) { PENDING("k3_mla_scratch"); return 0; }
void k3_mla_cached(float *out, const float *x, const K3MlaW *w, const K3Cfg *c, int T, float *scratch, float *kvc, float *ropec, int cached, int cap) { PENDING("k3_mla_cached"); }
void k3_mla(float *out, const float *x, const K3MlaW *w, const K3Cfg *c, int T, float *scratch) { PENDING("k3_mla"); }
size_t k3_moe_scratch(const K3Cfg *c) { PENDING("k3_moe_scratch"); return 0; }
void k3_moe(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T, int *idx, float *wt, float *scratch) { PENDING("k3_moe"); }
void k3_moe_prefill(float *out, const float *x, const K3MoeW *w, const K3Cfg *c, int T, int *idx, float *wt, float *scratch) { PENDING("k3_moe_prefill"); }
size_t k3_kda_scratch(const K3Cfg *c, int T) { PENDING("k3_kda_scratch"); return 0; }
void k3_kda_layer(float *out, const float *x, const K3KdaW *w, const K3Cfg *c, int T, float *state, float *scratch) { PENDING("k3_kda_layer"); }
size_t k3_layer_scratch(const K3Cfg *c, int T) { PENDING("k3_layer_scratch"); return 0; }
void k3_decoder_layer(float *h, float *br, int *nb, const K3LayerW *w, const K3Cfg *c, int li, int T, float *state, float *scratch) { PENDING("k3_decoder_layer"); }
void k3_decoder_layer_inc(float *h, float *br, int *nb, const K3LayerW *w, const K3Cfg *c, int li, int T, float *state, float *scratch, float *kvc, float *ropec, int cached, int cap) { PENDING("k3_decoder_layer_inc"); }

size_t k3d_mla_ws_bytes(const K3dMlaShape *s, int B, int cap) { PENDING("k3d_mla_ws_bytes"); return 0; }
int k3d_mla_decode(float *out, const float *x, const K3dMlaW *w, const K3dMlaShape *s, int B, uint16_t *cache, int cap, const int *pos, int accumulate, void *ws, size_t ws_bytes) { return PENDING("k3d_mla_decode"); }
K3dModel *k3d_model_create(const K3dStackCfg *cfg, uint64_t seed) { PENDING("k3d_model_create"); return nullptr; }
void k3d_model_destroy(K3dModel *m) {}
int k3d_model_fill_context(K3dModel *m, int len, uint64_t seed) { return PENDING("k3d_model_fill_context"); }
int k3d_model_step_dev(K3dModel *m, const int *ids, int *next_ids, float *logits) { return PENDING("k3d_model_step_dev"); }
int k3d_model_step_host(K3dModel *m, const int *ids_host, int *next_host) { return PENDING("k3d_model_step_host"); }
int k3d_model_use_graph(K3dModel *m, int on) { return PENDING("k3d_model_use_graph"); }
void *k3d_model_tensor(K3dModel *m, const char *name, size_t *bytes) { return nullptr; }
double k3d_model_last_step_bytes(K3dModel *m) { return 0.0; }

}
