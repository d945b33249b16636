"""The chunked (WY) form of the KDA recurrence, restated in numpy float64, against the
oracle's sequential k3_kda_step (k3_ops.c:186-243). This pins the algebra the chunk-64
prefill kernels implement (k3_kda.cu): cumulative log2 decays per chunk, L and M from
decay-weighted key products, forward substitution for U and W, then per chunk
X = U - W S, O = Qt S + M X and S = diag(2^G_last) S + Kb^T X. CPU only."""
import numpy as np
import pytest


def _chunked(S0, q, k, v, al, be, C=64):
    """S0 [H][dk][dv]; q, k, al [T][H][dk]; v [T][H][dv]; be [T][H]. Returns (S, o)."""
    T, H, dk = q.shape
    dv = v.shape[2]
    S = S0.astype(np.float64).copy()
    o = np.zeros((T, H, dv))
    for h in range(H):
        for c0 in range(0, T, C):
            n = min(C, T - c0)
            kk = np.zeros((C, dk)); qq = np.zeros((C, dk)); vv = np.zeros((C, dv))
            aa = np.ones((C, dk)); bb = np.zeros(C)
            kk[:n], qq[:n], vv[:n] = k[c0:c0 + n, h], q[c0:c0 + n, h], v[c0:c0 + n, h]
            aa[:n], bb[:n] = al[c0:c0 + n, h], be[c0:c0 + n, h]
            G = np.cumsum(np.maximum(np.log2(np.maximum(aa, 1e-300)), -126.0), axis=0)
            E = np.exp2(G[:, None, :] - G[None, :, :])              # [t][s][i]
            L = np.tril(np.einsum("ti,si,tsi->ts", kk, kk, E), -1)
            M = np.tril(np.einsum("ti,si,tsi->ts", qq, kk, E), 0)
            Kt, Qt = kk * np.exp2(G), qq * np.exp2(G)
            Kb, g_last = kk * np.exp2(G[-1] - G), np.exp2(G[-1])
            U = np.zeros((C, dv)); W = np.zeros((C, dk))
            for t in range(C):
                U[t] = bb[t] * (vv[t] - L[t, :t] @ U[:t])
                W[t] = bb[t] * (Kt[t] - L[t, :t] @ W[:t])
            X = U - W @ S[h]
            o[c0:c0 + n, h] = (Qt @ S[h] + M @ X)[:n]
            S[h] = g_last[:, None] * S[h] + Kb.T @ X
    return S, o


def _sequential(oracle, S0, q, k, v, al, be):
    S = S0.copy()
    o = np.zeros((q.shape[0], q.shape[1], v.shape[2]), np.float32)
    for t in range(q.shape[0]):
        S2, o2 = oracle.kda_decode(S[None], q[t][None], k[t][None], v[t][None], al[t][None],
                                   be[t][None])
        S, o[t] = S2[0], o2[0]
    return S, o


@pytest.mark.parametrize("T,H,dk,dv,decay", [(150, 2, 32, 16, (0.9, 1.0)),
                                             (70, 1, 16, 8, (0.05, 0.5)),
                                             (64, 1, 8, 8, (0.0, 1.0))])
def test_chunked_form_equals_sequential_step(oracle, T, H, dk, dv, decay):
    g = np.random.default_rng(T + dk)

    def unit(x):
        return (x / np.linalg.norm(x, axis=-1, keepdims=True)).astype(np.float32)

    S0 = (g.standard_normal((H, dk, dv)) * 0.01).astype(np.float32)
    q, k = unit(g.standard_normal((T, H, dk))), unit(g.standard_normal((T, H, dk)))
    v = g.standard_normal((T, H, dv)).astype(np.float32)
    al = g.uniform(*decay, (T, H, dk)).astype(np.float32)
    be = g.uniform(0, 1, (T, H)).astype(np.float32)
    Sc, oc = _chunked(S0, q, k, v, al, be)
    Ss, os_ = _sequential(oracle, S0, q, k, v, al, be)
    # float64 chunked algebra vs the fp32 sequential oracle: fp32 rounding only
    assert np.abs(oc - os_).max() <= 1e-4 * np.abs(os_).max()
    assert np.abs(Sc - Ss).max() <= 1e-4 * np.abs(Ss).max()
