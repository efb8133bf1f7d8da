"""CPU restatement of the reference's Gated DeltaNet token mixer (test infrastructure
only; parity unpinned: no golden vectors exist for this op in the reference and its
WGSL cannot run here, so the restatement follows the shader's text).

Follows crates/engine/src/shaders/deltanet.wgsl:80-160, per head h and token m:
  q, k, v = silu(causal depthwise conv of the last 3 inputs and this one)
  q = q / sqrt(|q|^2 + 1e-6) / sqrt(KD),  k = k / sqrt(|k|^2 + 1e-6)
  decay = exp(neg_a * softplus(a + dt_bias)),  beta = sigmoid(b)
  delta = (v - decay * S^T k) * beta,  o = decay * S^T q + delta * (k . q)
  S = decay * S + k delta^T
  o = o / sqrt(mean(o^2) + eps) * gate_norm * silu(z)
in float64.  State slots as the shader keeps them: the current slot `slot` is read;
without spec the final state goes back to it, with spec the state after token m goes
to slot (slot + 1 + m) % 3.

Layouts: proj f32 [M, C + NH VD + 2 NH] with C = NH (2 KD + VD), rows
[q (NH KD) | k (NH KD) | v (NH VD) | z (NH VD) | b (NH) | a (NH)];
conv_w f32 [C, 4] (taps, oldest first); conv_state f32 [3, C, 3]; state f32 [3, NH, KD, VD].
"""

import numpy as np

KD = VD = 128


def _silu(x):
    return x / (1.0 + np.exp(-x))


def deltanet(proj, conv_w, conv_state, state, neg_a, dt_bias, gate_norm, NH, m, slot, eps=1e-6, spec=False):
    """Returns (out f64 [m, NH VD], conv_state', state') with the slot updates applied."""
    C = NH * (2 * KD + VD)
    proj = np.asarray(proj, np.float64).reshape(m, -1)
    w = np.asarray(conv_w, np.float64).reshape(C, 4)
    cs = np.array(conv_state, np.float64).reshape(3, C, 3)
    st = np.array(state, np.float64).reshape(3, NH, KD, VD)
    win = cs[slot].copy()
    S = st[slot].copy()
    out = np.zeros((m, NH * VD))
    for t in range(m):
        x = proj[t, :C]
        y = _silu(w[:, 0] * win[:, 0] + w[:, 1] * win[:, 1] + w[:, 2] * win[:, 2] + w[:, 3] * x)
        win = np.concatenate([win[:, 1:], x[:, None]], axis=1)
        for h in range(NH):
            q = y[h * KD:(h + 1) * KD]
            k = y[NH * KD + h * KD: NH * KD + (h + 1) * KD]
            v = y[2 * NH * KD + h * VD: 2 * NH * KD + (h + 1) * VD]
            q = q / np.sqrt((q * q).sum() + 1e-6) / np.sqrt(KD)
            k = k / np.sqrt((k * k).sum() + 1e-6)
            b = proj[t, C + NH * VD + h]
            a = proj[t, C + NH * VD + NH + h] + dt_bias[h]
            sp = a if a > 20.0 else np.log1p(np.exp(a))
            decay = np.exp(neg_a[h] * sp)
            beta = 1.0 / (1.0 + np.exp(-b))
            sk = S[h].T @ k
            sq = S[h].T @ q
            delta = (v - decay * sk) * beta
            o = decay * sq + delta * (k @ q)
            S[h] = decay * S[h] + np.outer(k, delta)
            z = proj[t, C + h * VD: C + (h + 1) * VD]
            o = o / np.sqrt((o * o).mean() + eps) * gate_norm * _silu(z)
            out[t, h * VD:(h + 1) * VD] = o
        if spec:
            cs[(slot + 1 + t) % 3] = win
            st[(slot + 1 + t) % 3] = S
    if not spec:
        cs[slot] = win
        st[slot] = S
    return out, cs, st
