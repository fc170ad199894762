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
        norm(p + "attn_q_norm.weight", hd)
        norm(p + "attn_k_norm.weight", hd)
        q(p + "attn_q.weight", Q4_K, H * 2 * hd, c["hidden"])
        q(p + "attn_k.weight", Q4_K, KV * hd, c["hidden"])
        q(p + "attn_v.weight", Q4_K, KV * hd, c["hidden"])
        q(p + "attn_output.weight", Q4_K, c["hidden"], H * hd)
        q(p + "ffn_gate.weight", Q4_K, c["ffn"], c["hidden"])
        q(p + "ffn_up.weight", Q4_K, c["ffn"], c["hidden"])
        q(p + "ffn_down.weight", Q6_K, c["hidden"], c["ffn"])
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
            self.layers.append(dict(
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

    def _mv(self, qtype, w, k, x):
        return self.orc.matvec(qtype, w, k, self.orc.quantize_act(qtype, x[None]))[0]

    def step(self, token, pos):
        """Returns (local logits, hidden state before the output norm)."""
        orc, c, p = self.orc, self.c, self.p
        hd, D, eps = c["head_dim"], c["hidden"], c["rms_eps"]
        r0 = self.rank == 0
        h = orc.dequantize(self.qt["token_embd.weight"], self.embd[token:token + 1], D)[0]
        for Ly in self.layers:
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
            x2 = rms_scaled(h2, Ly["post_norm"], eps)
            g = self._mv(Ly["tg"], Ly["wg"], D, x2)
            u = self._mv(Ly["tg"], Ly["wu"], D, x2)
            a = orc.silu_mul(g, u)
            h = self._mv(Ly["td"], Ly["wd"], p["n_f"], a)
            if r0:
                h = h + h2
            h = self.allreduce(h)
        self.hidden = h
        logits = self._mv(self.qt["output.weight"], self.lmh, D, rms_scaled(h, self.out_norm, eps))
        return logits, h
