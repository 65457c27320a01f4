"""CPU ORACLE for LlamaModelInt8 (model/llama/forward_int8.rs:148-547).

TEST INFRASTRUCTURE ONLY (the checker of the GPU model; never imported by
the product).  Orchestrates the C++ restatements in ref_hotpath.cpp exactly
as the reference's block does:

  attn_sublayer (forward_int8.rs:265-289 / :325-348 for decode):
    normed = rmsnorm(x, attn_norm); q,k,v = proj_int8(normed, wq|wk|wv)
    rope(q), rope(k) at start_pos; attention (causal, offset start_pos)
    x = x + proj_int8(attn, wo)
  ffn_sublayer (:350-357):
    normed = rmsnorm(x, ffn_norm); h = swiglu(proj(normed, wgate), proj(normed, wup))
    x = x + proj_int8(h, wdown)
  model: embed -> blocks -> rmsnorm(output_norm) -> proj_int8(x, output)

proj_int8 is matmul_int8_from_f32 with per-tensor quantization of the whole
[seq, d] input (int8.rs:113-143).
"""
import numpy as np

import oracle


def tiny_config():
    """forward_int8.rs:559-572 (2 layers, d=16, 2 heads, ffn 32, ctx 64, vocab 32)."""
    return dict(n_layers=2, dim=16, n_heads=2, n_kv_heads=2, ffn_dim=32, vocab=32, max_seq=64,
                rope_base=10000.0, rms_eps=1e-5)


def smooth_model_weights(cfg):
    """make_int8_model (forward_int8.rs:583-621): smooth_weight matrices
    quantized per channel, unit norms."""
    d, V, ffn = cfg["dim"], cfg["vocab"], cfg["ffn_dim"]
    hd = d // cfg["n_heads"]
    qd, kvd = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd

    def q(rows, cols, seed):
        return oracle.quantize_per_channel(oracle.smooth_weight(rows, cols, seed), rows, cols)

    layers = []
    for i in range(cfg["n_layers"]):
        s = float(i + 1)
        layers.append(dict(wq=q(qd, d, s * 1.0), wk=q(kvd, d, s * 1.1), wv=q(kvd, d, s * 1.2),
                           wo=q(d, qd, s * 1.3), wgate=q(ffn, d, s * 1.4), wup=q(ffn, d, s * 1.5),
                           wdown=q(d, ffn, s * 1.6)))
    return dict(token_embd=oracle.smooth_weight(V, d, 0.5), layers=layers,
                attn_norm=np.ones(cfg["n_layers"] * d, np.float32),
                ffn_norm=np.ones(cfg["n_layers"] * d, np.float32),
                output_norm=np.ones(d, np.float32), output=q(V, d, 0.7))


def _rmsnorm64(x, d, w, eps):
    """rmsnorm (ops/norm/rmsnorm.rs:51-117) with the mean square accumulated
    in float64: the same formula in another rounding order."""
    x = np.asarray(x, np.float32).reshape(-1, d)
    ms = (x.astype(np.float64) ** 2).mean(axis=1).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    return (np.asarray(w, np.float32)[None, :] * (x * inv[:, None])).astype(np.float32).reshape(-1)


def _gqa64(q, k, v, seq_q, seq_k, n_heads, n_kv, hd, start_pos):
    """Causal GQA attention with the cache offset (attention/gqa.rs:217-237)
    with scores, softmax and the weighted sum in float64."""
    q = np.asarray(q, np.float32).reshape(seq_q, n_heads, hd).astype(np.float64)
    k = np.asarray(k, np.float32).reshape(seq_k, n_kv, hd).astype(np.float64)
    v = np.asarray(v, np.float32).reshape(seq_k, n_kv, hd).astype(np.float64)
    group = n_heads // n_kv
    mask = np.arange(seq_k)[None, :] > (start_pos + np.arange(seq_q))[:, None]
    out = np.empty((seq_q, n_heads, hd))
    for h in range(n_heads):
        s = (q[:, h, :] @ k[:, h // group, :].T) / np.sqrt(hd)
        s[mask] = -np.inf
        s = np.exp(s - s.max(axis=1, keepdims=True))
        out[:, h, :] = (s / s.sum(axis=1, keepdims=True)) @ v[:, h // group, :]
    return out.astype(np.float32).reshape(-1)


def _swiglu64(gate, up):
    g = np.asarray(gate, np.float32).astype(np.float64)
    return (g / (1.0 + np.exp(-g)) * np.asarray(up, np.float32)).astype(np.float32).reshape(-1)


class LlamaInt8Oracle:
    """proj="par" (default): projections as proj_int8_par (the AVX2 row-parallel
    product); proj="scalar": as proj_int8, the scalar matmul_int8_from_f32
    that the reference's decode step calls (forward_int8.rs:333-346).  Both
    give the same numbers.

    glue="reference" (default): the reference's f32 glue, restated op by
    op.  glue="f64": the same model with RMSNorm, attention and SwiGLU
    accumulated in float64 and rounded to f32 — the same mathematics in
    another rounding order.  The projections (the INT8 products) are the
    reference's in both.  The tests use the second to measure how far two
    correct f32 implementations drift apart through the per-tensor INT8
    activation quantization (a 1-ulp change of an activation can move its
    INT8 code), which sets the model-level tolerance."""

    def __init__(self, cfg, w, glue="reference", proj="par"):
        assert glue in ("reference", "f64") and proj in ("par", "scalar")
        self.glue, self.proj = glue, proj
        self.cfg, self.w = cfg, w
        self.hd = cfg["dim"] // cfg["n_heads"]
        self.cos, self.sin = oracle.rope_table(cfg["max_seq"], self.hd, cfg["rope_base"])
        L, S, kvd = cfg["n_layers"], cfg["max_seq"], cfg["n_kv_heads"] * self.hd
        self.kc = np.zeros((L, S, kvd), np.float32)   # KvCache (cache/kv_cache.rs:44-72)
        self.vc = np.zeros((L, S, kvd), np.float32)

    def _proj(self, x, rows, wpair, n_out):
        """proj_int8_par (forward_int8.rs:87-96): quantize_symmetric over the
        whole [rows, k] input, then matmul_int8_parallel; the same numbers as
        proj_int8 (:72-84), in the time the model-sized checks need."""
        data, scales = wpair
        k = x.size // rows
        if self.proj == "scalar":  # proj_int8 (:72-74): matmul_int8_from_f32, scalar loop
            return oracle.matmul_int8_from_f32(x, rows, k, data, scales, n_out, k).reshape(-1)
        aq, s = oracle.quantize_symmetric(x)
        return oracle.matmul_int8_parallel(aq, s, data, scales, n_out, k, rows).reshape(-1)

    def _block(self, li, x, seq, start_pos, use_cache):
        c, lw = self.cfg, self.w["layers"][li]
        d, H, Hkv, hd, ffn = c["dim"], c["n_heads"], c["n_kv_heads"], self.hd, c["ffn_dim"]
        qd, kvd = H * hd, Hkv * hd
        f64 = self.glue == "f64"
        rmsnorm = _rmsnorm64 if f64 else oracle.rmsnorm
        gqa = _gqa64 if f64 else oracle.gqa_causal_offset
        normed = rmsnorm(x, d, self.w["attn_norm"][li * d:(li + 1) * d], c["rms_eps"])
        q = self._proj(normed, seq, lw["wq"], qd)
        k = self._proj(normed, seq, lw["wk"], kvd)
        v = self._proj(normed, seq, lw["wv"], kvd)
        q = oracle.rope_apply(q, seq, H, hd, self.cos, self.sin, start_pos)
        k = oracle.rope_apply(k, seq, Hkv, hd, self.cos, self.sin, start_pos)
        if use_cache:
            self.kc[li, start_pos:start_pos + seq] = k.reshape(seq, kvd)
            self.vc[li, start_pos:start_pos + seq] = v.reshape(seq, kvd)
            total = start_pos + seq
            attn = gqa(q, self.kc[li, :total], self.vc[li, :total], seq, total, H, Hkv, hd, start_pos)
        else:
            attn = gqa(q, k, v, seq, seq, H, Hkv, hd, start_pos)
        x = (x + self._proj(attn, seq, lw["wo"], d)).astype(np.float32)
        normed = rmsnorm(x, d, self.w["ffn_norm"][li * d:(li + 1) * d], c["rms_eps"])
        gate = self._proj(normed, seq, lw["wgate"], ffn)
        up = self._proj(normed, seq, lw["wup"], ffn)
        h = _swiglu64(gate, up) if f64 else oracle.swiglu(gate, up)
        return (x + self._proj(h, seq, lw["wdown"], d)).astype(np.float32)

    def _head(self, x, seq):
        c = self.cfg
        rmsnorm = _rmsnorm64 if self.glue == "f64" else oracle.rmsnorm
        x = rmsnorm(x, c["dim"], self.w["output_norm"], c["rms_eps"])
        return self._proj(x, seq, self.w["output"], c["vocab"]).reshape(seq, c["vocab"])

    def _embed(self, tokens):
        d = self.cfg["dim"]
        for t in tokens:
            if t >= self.cfg["vocab"]:
                raise ValueError(f"token id {t} >= vocab_size {self.cfg['vocab']}")
        emb = np.asarray(self.w["token_embd"], np.float32).reshape(-1, d)
        return emb[np.asarray(tokens, np.int64)].reshape(-1).copy()

    def forward(self, tokens):
        """forward_int8.rs:516-529 (no cache, start_pos 0)."""
        if len(tokens) == 0:
            raise ValueError("forward: token list must not be empty")
        x = self._embed(tokens)
        for li in range(self.cfg["n_layers"]):
            x = self._block(li, x, len(tokens), 0, use_cache=False)
        return self._head(x, len(tokens))

    def prefill_cached(self, tokens):
        """Cached prefill at start_pos 0 (the model-level addition)."""
        return self.forward_cached(tokens, 0)

    def forward_cached(self, tokens, start_pos):
        """Every block's forward_cached (forward_int8.rs:206-215) at
        start_pos, which forward_cached_parallel (:232-249) equals, then the
        output norm and head."""
        x = self._embed(tokens)
        for li in range(self.cfg["n_layers"]):
            x = self._block(li, x, len(tokens), start_pos, use_cache=True)
        return self._head(x, len(tokens))

    def block_forward(self, li, x, start_pos):
        """TransformerBlockInt8::forward_cached (forward_int8.rs:206-215) of
        layer li on x [seq, d] with this oracle's cache."""
        x = np.asarray(x, np.float32).reshape(-1)
        seq = x.size // self.cfg["dim"]
        return self._block(li, x, seq, start_pos, use_cache=True).reshape(seq, self.cfg["dim"])

    def forward_decode(self, token, pos):
        """forward_int8.rs:538-546."""
        x = self._embed([token])
        for li in range(self.cfg["n_layers"]):
            x = self._block(li, x, 1, pos, use_cache=True)
        return self._head(x, 1)[0]
