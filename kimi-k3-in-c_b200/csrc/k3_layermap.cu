// k3_layermap.cu -- host-only pieces of include/k3/k3.h: the layer map (k3_ops.c:84-91,
// full_attn is one-based) and the expert-drop counter (k3.h:384-388).
#include "k3_common.cuh"

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

}  // extern "C"
