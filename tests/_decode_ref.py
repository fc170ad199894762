"""Decode-step reference for the engine tests (test helper, CPU only).

Composes the oracle's ggml-semantics pieces (q8_K activation quantization,
vec_dot matvecs, dequant) with fp32 numpy glue into one decode step of the
attention-shaped model the engine runs (reference decode layer,
src/mono27b_executor.cu:2372-2479 for attention, :2475-2479 / :2564-2569 for
the FFN, :2577-2593 for the head):

  h   = dequant(token_embd[token])
  per layer:
    xq  = q8_K(RMSNorm(h) * attn_norm)
    q|g = attn_q . xq  (per head: hd query rows, then hd gate rows)
    k,v = attn_k . xq, attn_v . xq
    q,k = RoPE(RMSNorm_head(q|k) * q_norm|k_norm)       (neox pairs over n_rot)
    o   = softmax(q.K^T / sqrt(hd)) V                    (all cached positions)
    h2  = attn_output . q8_K(o * sigmoid(g)) + h
    h   = ffn_down . q8_K(silu(ffn_gate . x2) * (ffn_up . x2)) + h2,
          x2 = q8_K(RMSNorm(h2) * post_attention_norm)
  logits = output . q8_K(RMSNorm(h) * output_norm); next = first argmax

Hybrid models (attn_interval > 0: layer il is attention iff (il + 1) %
attn_interval == 0, reference src/mono27b_executor.cu:2372) run every other
layer as the Gated DeltaNet block of :2484-2548 (single GPU):

  x    = RMSNorm(h) * attn_norm
  c    = attn_qkv . x  (conv channels: q [ng][dk] | k [ng][dk] | v [dr][dv])
  z    = attn_gate . x ;  b, a = ssm_beta . x, ssm_alpha . x   (f16 weights: fp32 x)
  beta = sigmoid(b) ;  g = softplus(a + dt_bias) * ssm_a          (:816-826)
  c    = silu(causal conv over the last conv_kern inputs)         (:1488-1501)
  q, k = L2-normalised per group (sum of squares in fp64)         (:1118-1133)
  per value head j (group j % ng), state S_j [dv][dk]:            (:1526-1603)
    kv = S_j k ;  d = (v_j - e^g kv) * beta ;  S_j = e^g S_j + d k^T
    o_j = (S_j q) / sqrt(dk)
  y    = RMSNorm_j(o_j) * ssm_norm * silu(z_j)                   (:735-765)
  h2   = ssm_out . q8_K(y) + h, then the FFN as above

`RefDecoder(model, cfg, part)` computes the slice one tensor-parallel rank
holds: its query heads and the kv heads they use, its FFN rows, and its
vocabulary rows; o_proj / down then give partial sums that an `allreduce`
callback adds up (rank 0 adds the residual), exactly the split the engine
makes.  With the whole-model partition it is the plain single-GPU reference.
"""
import numpy as np

from _data import Q4_K, Q6_K, gauss_weights

F32 = 0
BLOCK = {Q4_K: (256, 144), Q6_K: (256, 210), 8: (32, 34), 13: (256, 176), 23: (256, 136)}

TINY = dict(n_layers=2, hidden=512, ffn=1024, n_head=4, n_kv_head=2, head_dim=128, vocab=1000, n_rot=64,
            rope_theta=1e7, rms_eps=1e-6)


F16 = 1


def is_attention(c, il):
    k = c.get("attn_interval", 0)
    return k == 0 or (il + 1) % k == 0


def ssm_dims(c):
    ng, dk, dr = c["ssm_n_group"], c["ssm_d_state"], c["ssm_dt_rank"]
    dv = c["ssm_d_inner"] // dr
    return ng, dk, dr, dv, c["ssm_d_inner"] + 2 * ng * dk, c["ssm_conv_kern"]


def delta_rule(S, q, k, v, beta, g):
    """One gated delta-rule step on a value head's state S [dv][dk] (fp32,
    updated in place), reference src/mono27b_executor.cu:1559-1589:
    kv = S k; d = (v - e^g kv) * beta; S = e^g S + d k^T; returns (S q) / sqrt(dk)."""
    f32 = np.float32
    gv = np.exp(f32(g)).astype(f32)
    kv = (S.astype(np.float64) @ k.astype(np.float64)).astype(f32)
    d = ((v - gv * kv) * f32(beta)).astype(f32)
    S[:] = (gv * S + d[:, None] * k[None, :]).astype(f32)
    return (S.astype(np.float64) @ q.astype(np.float64) / np.sqrt(S.shape[1])).astype(f32)


def make_model(orc, c, seed=0, sigma=0.02, norm_jitter=0.1, qtype=None, types=None):
    """name -> (ggml_type, row_elems, row_count, array): GGUF-named tensors of
    N(0, sigma^2) weights quantized by the oracle (the q4_k_m mix, or every
    matrix as `qtype`, e.g. q8_0 for a draft; `types` maps a layer tensor's
    short name, e.g. "ffn_down", to its type), norms 1 + N(0, jitter^2)."""
    rng = np.random.default_rng(seed)
    hd, H, KV = c["head_dim"], c["n_head"], c["n_kv_head"]
    t = {}
    s = [seed * 1000]
    types = types or {}

    def q(name, qt, rows, k):
        s[0] += 1
        short = name.split(".")[-2] if name.startswith("blk.") else None
        qt = types.get(short, qtype or qt)
        t[name] = (qt, k, rows, gauss_weights(orc, qt, rows, k, s[0], sigma))

    def norm(name, n):
        t[name] = (F32, n, 1, (1.0 + norm_jitter * rng.standard_normal(n)).astype(np.float32))

    q("token_embd.weight", Q4_K, c["vocab"], c["hidden"])
    q("output.weight", Q6_K, c["vocab"], c["hidden"])
    norm("output_norm.weight", c["hidden"])
    for l in range(c["n_layers"]):
        p = f"blk.{l}."
        norm(p + "attn_norm.weight", c["hidden"])
        norm(p + "post_attention_norm.weight", c["hidden"])
        q(p + "ffn_gate.weight", Q4_K, c["ffn"], c["hidden"])
        q(p + "ffn_up.weight", Q4_K, c["ffn"], c["hidden"])
        q(p + "ffn_down.weight", Q6_K, c["hidden"], c["ffn"])
        if not is_attention(c, l):
            ng, dk, dr, dv, cc, K = ssm_dims(c)
            q(p + "attn_qkv.weight", Q4_K, cc, c["hidden"])
            q(p + "attn_gate.weight", Q4_K, c["ssm_d_inner"], c["hidden"])
            q(p + "ssm_beta.weight", F16, dr, c["hidden"])
            q(p + "ssm_alpha.weight", F16, dr, c["hidden"])
            cw = (0.3 * rng.standard_normal((cc, K))).astype(np.float32)
            if types.get("ssm_conv1d") == F16:
                t[p + "ssm_conv1d.weight"] = (F16, K, cc, cw.astype(np.float16))
            else:
                t[p + "ssm_conv1d.weight"] = (F32, K, cc, cw)
            t[p + "ssm_dt.bias"] = (F32, dr, 1, (0.5 * rng.standard_normal(dr)).astype(np.float32))
            t[p + "ssm_a"] = (F32, dr, 1, (-np.exp(0.5 * rng.standard_normal(dr))).astype(np.float32))
            norm(p + "ssm_norm.weight", dv)
            q(p + "ssm_out.weight", Q4_K, c["hidden"], c["ssm_d_inner"])
            continue
        norm(p + "attn_q_norm.weight", hd)
        norm(p + "attn_k_norm.weight", hd)
        q(p + "attn_q.weight", Q4_K, H * 2 * hd, c["hidden"])
        q(p + "attn_k.weight", Q4_K, KV * hd, c["hidden"])
        q(p + "attn_v.weight", Q4_K, KV * hd, c["hidden"])
        q(p + "attn_output.weight", Q4_K, c["hidden"], H * hd)
    return t


def full_partition(c):
    return dict(q_lo=0, n_q=c["n_head"], kv_lo=0, n_kv=c["n_kv_head"], f_lo=0, n_f=c["ffn"], v_lo=0, n_v=c["vocab"])


def col_slice(qtype, w, k0, nk):
    """Columns [k0, k0+nk) of a quantized matrix (whole blocks)."""
    be, bb = BLOCK[qtype]
    assert k0 % be == 0 and nk % be == 0
    return np.ascontiguousarray(w[:, k0 // be * bb:(k0 + nk) // be * bb])


def rms_scaled(x, w, eps):
    x = np.asarray(x, dtype=np.float32)
    ms = np.float32(np.sum(x.astype(np.float64) ** 2) / x.size)
    return (x * (np.float32(1.0) / np.sqrt(ms + np.float32(eps)))) * w


def q8K_tie_margin(x):
    """Smallest distance of a q8_K code's unrounded value x * (-127 / max) to
    a rounding tie (k + 0.5), relative to max(|value|, 1), over the 256-value
    blocks of the fp32 vector x (ggml's quantize_row_q8_K rounds that value to
    nearest).  Another fp32 summation order moves an activation by a few ulps:
    a margin below ~1e-6 means the code may come out the other way."""
    best = np.inf
    x = np.asarray(x, dtype=np.float32).reshape(-1, 256)
    for blk in x:
        mx = blk[np.argmax(np.abs(blk))]
        if mx == 0:
            continue
        v = ((np.float32(-127.0) / mx) * blk).astype(np.float32)
        best = min(best, float((np.abs(v - np.floor(v) - 0.5) / np.maximum(np.abs(v), 1)).min()))
    return best


def rope(x, pos, n_rot, theta):
    half = n_rot // 2
    p = np.arange(half, dtype=np.float64)
    ang = pos * theta ** (-2.0 * p / n_rot)
    cs, sn = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    out = x.copy()
    a, b = x[:half], x[half:n_rot]
    out[:half] = a * cs - b * sn
    out[half:n_rot] = a * sn + b * cs
    return out


class RefDecoder:
    def __init__(self, orc, model, c, part=None, rank=0, allreduce=None, max_ctx=64):
        self.orc, self.c = orc, c
        self.p = part or full_partition(c)
        self.rank = rank
        self.allreduce = allreduce or (lambda v: v)
        p, hd = self.p, c["head_dim"]
        self.Gg = c["n_head"] // c["n_kv_head"]
        self.qt = {n: v[0] for n, v in model.items()}
        self.embd = model["token_embd.weight"][3]
        self.lmh = np.ascontiguousarray(model["output.weight"][3][p["v_lo"]:p["v_lo"] + p["n_v"]])
        self.out_norm = model["output_norm.weight"][3]
        self.layers = []
        for l in range(c["n_layers"]):
            g = lambda n: model[f"blk.{l}.{n}.weight"][3]
            tq = lambda n: model[f"blk.{l}.{n}.weight"][0]
            if not is_attention(c, l):
                assert self.rank == 0 and p == full_partition(c), "hybrid layers: single GPU"
                ng, dk, dr, dv, cc, K = ssm_dims(c)
                self.layers.append(dict(
                    ssm=True, attn_norm=g("attn_norm"), post_norm=g("post_attention_norm"),
                    t_qkv=tq("attn_qkv"), w_qkv=g("attn_qkv"), t_gate=tq("attn_gate"), w_gate=g("attn_gate"),
                    t_beta=tq("ssm_beta"), w_beta=g("ssm_beta"), t_alpha=tq("ssm_alpha"), w_alpha=g("ssm_alpha"),
                    conv_w=g("ssm_conv1d").astype(np.float32), dt_bias=model[f"blk.{l}.ssm_dt.bias"][3],
                    ssm_a=model[f"blk.{l}.ssm_a"][3], ssm_norm=g("ssm_norm"), t_out=tq("ssm_out"), w_out=g("ssm_out"),
                    tg=tq("ffn_gate"), td=tq("ffn_down"), wg=g("ffn_gate"), wu=g("ffn_up"), wd=g("ffn_down"),
                    conv=np.zeros((cc, K - 1), np.float32), S=np.zeros((dr, dv, dk), np.float32)))
                continue
            self.layers.append(dict(ssm=False, 
                tqkv=tq("attn_q"), to=tq("attn_output"), tg=tq("ffn_gate"), td=tq("ffn_down"),
                attn_norm=g("attn_norm"), post_norm=g("post_attention_norm"), q_norm=g("attn_q_norm"),
                k_norm=g("attn_k_norm"),
                wq=np.ascontiguousarray(g("attn_q")[p["q_lo"] * 2 * hd:(p["q_lo"] + p["n_q"]) * 2 * hd]),
                wk=np.ascontiguousarray(g("attn_k")[p["kv_lo"] * hd:(p["kv_lo"] + p["n_kv"]) * hd]),
                wv=np.ascontiguousarray(g("attn_v")[p["kv_lo"] * hd:(p["kv_lo"] + p["n_kv"]) * hd]),
                wo=col_slice(tq("attn_output"), g("attn_output"), p["q_lo"] * hd, p["n_q"] * hd),
                wg=np.ascontiguousarray(g("ffn_gate")[p["f_lo"]:p["f_lo"] + p["n_f"]]),
                wu=np.ascontiguousarray(g("ffn_up")[p["f_lo"]:p["f_lo"] + p["n_f"]]),
                wd=col_slice(tq("ffn_down"), g("ffn_down"), p["f_lo"], p["n_f"]),
                kc=np.zeros((max_ctx, p["n_kv"], hd), np.float32), vc=np.zeros((max_ctx, p["n_kv"], hd), np.float32)))
        self.hidden = None
        self.tie_margin = np.inf  # q8K_tie_margin over the last step's q8_K activations

    def _mv(self, qtype, w, k, x):
        if self.orc.act_type_for(qtype) == self.orc.Q8_K:
            self.tie_margin = min(self.tie_margin, q8K_tie_margin(x))
        return self.orc.matvec(qtype, w, k, self.orc.quantize_act(qtype, x[None]))[0]

    def _ffn(self, Ly, h2, p, r0):
        """RMSNorm -> gate/up SwiGLU -> down (+ residual on rank 0), summed over ranks."""
        D, eps = self.c["hidden"], self.c["rms_eps"]
        x2 = rms_scaled(h2, Ly["post_norm"], eps)
        g = self._mv(Ly["tg"], Ly["wg"], D, x2)
        u = self._mv(Ly["tg"], Ly["wu"], D, x2)
        a = self.orc.silu_mul(g, u)
        h = self._mv(Ly["td"], Ly["wd"], p["n_f"], a)
        if r0:
            h = h + h2
        return self.allreduce(h)

    def _ssm(self, Ly, h):
        """The Gated DeltaNet block (reference src/mono27b_executor.cu:2484-2548): h -> h2."""
        c = self.c
        D, eps = c["hidden"], c["rms_eps"]
        ng, dk, dr, dv, cc, K = ssm_dims(c)
        f32 = np.float32
        silu = lambda v: (v / (f32(1) + np.exp(-v))).astype(f32)
        x = rms_scaled(h, Ly["attn_norm"], eps)
        qkv = self._mv(Ly["t_qkv"], Ly["w_qkv"], D, x)
        z = self._mv(Ly["t_gate"], Ly["w_gate"], D, x)
        braw = self._mv(Ly["t_beta"], Ly["w_beta"], D, x)
        araw = self._mv(Ly["t_alpha"], Ly["w_alpha"], D, x)
        beta = (f32(1) / (f32(1) + np.exp(-braw))).astype(f32)
        zz = (araw + Ly["dt_bias"]).astype(f32)
        sp = np.where(zz > 20, zz, np.log(f32(1) + np.exp(np.minimum(zz, 20)))).astype(f32)
        g = (sp * Ly["ssm_a"]).astype(f32)
        # causal conv, state oldest first (:1488-1501)
        st, w = Ly["conv"], Ly["conv_w"]
        s = ((st * w[:, :K - 1]).sum(1) + qkv * w[:, K - 1]).astype(f32)
        st[:, :-1] = st[:, 1:]
        st[:, -1] = qkv
        cv = silu(s)

        def l2(a):
            ss = (a.astype(np.float64) ** 2).sum(1).astype(f32)
            return (a * (f32(1) / np.sqrt(np.maximum(ss, f32(eps) * f32(eps))))[:, None]).astype(f32)

        q = l2(cv[:ng * dk].reshape(ng, dk))
        k = l2(cv[ng * dk:2 * ng * dk].reshape(ng, dk))
        v = cv[2 * ng * dk:].reshape(dr, dv)
        o = np.empty((dr, dv), f32)
        for j in range(dr):
            gi = j % ng  # value head j reads q/k group j % ng
            o[j] = delta_rule(Ly["S"][j], q[gi], k[gi], v[j], beta[j], g[j])
        zs = silu(z)
        y = np.concatenate([rms_scaled(o[j], Ly["ssm_norm"], eps) * zs[j * dv:(j + 1) * dv] for j in range(dr)])
        return self._mv(Ly["t_out"], Ly["w_out"], c["ssm_d_inner"], y.astype(f32)) + h

    def step(self, token, pos):
        """Returns (local logits, hidden state before the output norm)."""
        orc, c, p = self.orc, self.c, self.p
        self.tie_margin = np.inf
        hd, D, eps = c["head_dim"], c["hidden"], c["rms_eps"]
        r0 = self.rank == 0
        h = orc.dequantize(self.qt["token_embd.weight"], self.embd[token:token + 1], D)[0]
        for Ly in self.layers:
            if Ly["ssm"]:
                h2 = self._ssm(Ly, h)
                h = self._ffn(Ly, h2, p, r0)
                continue
            x = rms_scaled(h, Ly["attn_norm"], eps)
            qg = self._mv(Ly["tqkv"], Ly["wq"], D, x)
            kk = self._mv(Ly["tqkv"], Ly["wk"], D, x)
            vv = self._mv(Ly["tqkv"], Ly["wv"], D, x)
            for j in range(p["n_kv"]):
                kh = rms_scaled(kk[j * hd:(j + 1) * hd], Ly["k_norm"], eps)
                Ly["kc"][pos, j] = rope(kh, pos, c["n_rot"], c["rope_theta"])
                Ly["vc"][pos, j] = vv[j * hd:(j + 1) * hd]
            o = np.empty(p["n_q"] * hd, np.float32)
            gate = np.empty(p["n_q"] * hd, np.float32)
            for hh in range(p["n_q"]):
                j = (p["q_lo"] + hh) // self.Gg - p["kv_lo"]
                qh = rms_scaled(qg[hh * 2 * hd:hh * 2 * hd + hd], Ly["q_norm"], eps)
                qh = rope(qh, pos, c["n_rot"], c["rope_theta"])
                gate[hh * hd:(hh + 1) * hd] = qg[hh * 2 * hd + hd:(hh + 1) * 2 * hd]
                K = Ly["kc"][:pos + 1, j].astype(np.float64)
                V = Ly["vc"][:pos + 1, j].astype(np.float64)
                sc = K @ qh.astype(np.float64) / np.sqrt(hd)
                w = np.exp(sc - sc.max())
                o[hh * hd:(hh + 1) * hd] = (w @ V / w.sum()).astype(np.float32)
            og = (o * (np.float32(1.0) / (np.float32(1.0) + np.exp(-gate)))).astype(np.float32)
            h2 = self._mv(Ly["to"], Ly["wo"], p["n_q"] * hd, og)
            if r0:
                h2 = h2 + h
            h2 = self.allreduce(h2)
            h = self._ffn(Ly, h2, p, r0)
        self.hidden = h
        logits = self._mv(self.qt["output.weight"], self.lmh, D, rms_scaled(h, self.out_norm, eps))
        return logits, h
