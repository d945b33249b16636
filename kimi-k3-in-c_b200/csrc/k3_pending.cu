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


}
