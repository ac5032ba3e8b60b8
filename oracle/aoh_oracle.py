"""CPU oracle for the head-mixed attention runtime and the effective-rank classifier.

TEST INFRASTRUCTURE ONLY.  This module restates, in numpy, the algorithm of the
reference implementation (ernie-research/AoH) for the path the CUDA library
replaces.  Only the tests, the smoke check and the CPU-baseline leg of the
benchmark may import it, and only as the checker / the timed CPU reference --
the product path never calls it.

Parity of this restatement is PINNED against outputs of the reference itself:
``tests/golden/make_golden.py`` imports the reference's own modules, drives
them on seeded inputs and stores the results under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this module against every fixture.

Each function cites the reference lines it restates (paths are relative to the
reference project root).

Numerics follow the reference's eager path:
  * scores are float32 products of float32-upcast q and k, times ``D ** -0.5``
    (eval/efficiency/benchmark_llama31.py:127, attention_utils.py:116);
  * masked scores are ``finfo(float32).min`` (benchmark_llama31.py:131,
    attention_utils.py:117);
  * softmax in float32, probabilities cast to the input dtype before P.V
    (benchmark_llama31.py:132, attention_utils.py:118);
  * P.V accumulates in float32 and the output is rounded to the input dtype.
bfloat16 tensors are represented as float32 arrays holding bf16 values.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

F32 = np.float32
_NEG = np.finfo(np.float32).min
EPS = 1e-12  # aoh/effective_rank.py:24


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bfloat16 (ties to even), as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((u + bias) & np.uint32(0xFFFF0000)).view(np.float32)


def _to_dtype(x: np.ndarray, dtype: str) -> np.ndarray:
    return bf16_round(x) if dtype == "bf16" else x.astype(F32, copy=False)


# ----------------------------------------------------------------------------
# attention primitives
# ----------------------------------------------------------------------------

def repeat_kv(x: np.ndarray, n_rep: int) -> np.ndarray:
    """(B,G,S,D) -> (B,G*n_rep,S,D); eval/efficiency/benchmark_llama31.py:108-113."""
    if n_rep == 1:
        return x
    return np.repeat(x, n_rep, axis=1)


def causal_mask(q_len: int, k_len: int, past_len: int) -> np.ndarray:
    """True = allowed; benchmark_llama31.py:116-120."""
    q_pos = np.arange(past_len, past_len + q_len)[:, None]
    k_pos = np.arange(k_len)[None, :]
    return k_pos <= q_pos


def _softmax_f32(scores: np.ndarray) -> np.ndarray:
    m = scores.max(axis=-1, keepdims=True)
    e = np.exp(scores - m, dtype=F32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)


def _pv(probs: np.ndarray, v: np.ndarray, dtype: str) -> np.ndarray:
    probs = _to_dtype(probs, dtype)
    out = np.matmul(probs, v.astype(F32, copy=False))
    return _to_dtype(out, dtype)


def eager_attention(q, k, v, past_len: int, causal: bool, dtype: str) -> np.ndarray:
    """Retrieval-head attention; benchmark_llama31.py:123-132 (benchmark_qwen.py:132-141).

    q (B,H,Q,D), k/v (B,H,S,D) (already GQA-expanded) -> (B,H,Q,D)."""
    scale = F32(q.shape[-1] ** -0.5)
    scores = np.matmul(q.astype(F32), np.swapaxes(k.astype(F32), -1, -2)) * scale
    if causal:
        mask = causal_mask(q.shape[-2], k.shape[-2], past_len)
        scores = np.where(mask[None, None], scores, _NEG).astype(F32)
    return _pv(_softmax_f32(scores), v, dtype)


def cached_positions(past_len: int, cached_len: int, sink_size: int) -> np.ndarray:
    """Positions of a streaming head's cached keys; attention_utils.py:7-20."""
    if cached_len == past_len:
        return np.arange(past_len)
    sink_len = min(sink_size, cached_len)
    recent_len = cached_len - sink_len
    parts = [np.arange(sink_len)]
    if recent_len:
        parts.append(np.arange(past_len - recent_len, past_len))
    return np.concatenate(parts)


def streaming_attention(q, k, v, *, past_len: int, cached_len: int, sink_size: int,
                        recent_size: int, dtype: str) -> np.ndarray:
    """Sink + recent-window attention; attention_utils.py:92-119."""
    query_len = q.shape[-2]
    old_pos = cached_positions(past_len, cached_len, sink_size)
    new_pos = np.arange(past_len, past_len + query_len)
    key_pos = np.concatenate([old_pos, new_pos])
    causal = key_pos[None, :] <= new_pos[:, None]
    sink = key_pos[None, :] < sink_size
    recent = key_pos[None, :] >= (new_pos[:, None] - recent_size)
    allowed = causal & (sink | recent)
    scale = F32(q.shape[-1] ** -0.5)
    scores = np.matmul(q.astype(F32), np.swapaxes(k.astype(F32), -1, -2)) * scale
    scores = np.where(allowed[None, None], scores, _NEG).astype(F32)
    return _pv(_softmax_f32(scores), v, dtype)


def compress_stream(k, v, sink_size: int, recent_size: int):
    """Keep the first ``sink`` and last ``recent`` tokens; attention_utils.py:23-42."""
    budget = sink_size + recent_size
    if k.shape[2] <= budget:
        return k.copy(), v.copy()
    kp, vp = [], []
    if sink_size:
        kp.append(k[:, :, :sink_size]); vp.append(v[:, :, :sink_size])
    if recent_size:
        kp.append(k[:, :, -recent_size:]); vp.append(v[:, :, -recent_size:])
    if not kp:
        return k[:, :, :0].copy(), v[:, :, :0].copy()
    return np.concatenate(kp, axis=2), np.concatenate(vp, axis=2)


def head_permutation(labels_row: np.ndarray, num_q: int, num_kv: int):
    """Retrieval KV groups first, then streaming; eval/efficiency/reorder_weights.py:40-48."""
    grp = num_q // num_kv
    retrieval_kv = np.where(labels_row >= 0.5)[0]
    streaming_kv = np.where(labels_row < 0.5)[0]
    kv_perm = np.concatenate([retrieval_kv, streaming_kv]).astype(np.int64)
    q_perm = np.concatenate([np.arange(g * grp, (g + 1) * grp) for g in kv_perm]).astype(np.int64)
    return kv_perm, q_perm


# ----------------------------------------------------------------------------
# per-layer runtime: AoHKVCache + patched forward, without the projections
# ----------------------------------------------------------------------------

@dataclass
class OracleKVCache:
    """AoHKVCache restated; eval/efficiency/benchmark_llama31.py:135-184.

    Heads are kept in the reference's reordered (retrieval-first) order; the
    per-layer permutation comes from the labels."""
    num_layers: int
    labels: np.ndarray            # (L, G), 1 = retrieval
    sink_size: int
    recent_size: int
    dtype: str = "f32"
    kv_seq_len: int = 0
    # "eager" or "flash" (the decoding-simulation protocol, attention_utils.py:45-89)
    backend: str = "eager"
    full_k: list = field(default_factory=list)
    full_v: list = field(default_factory=list)
    stream_k: list = field(default_factory=list)
    stream_v: list = field(default_factory=list)

    def __post_init__(self):
        if self.sink_size < 0 or self.recent_size < 0:  # benchmark_llama31.py:257-258
            raise ValueError("sink_size and recent_size must be non-negative")
        L = self.num_layers
        self.full_k, self.full_v = [None] * L, [None] * L
        self.stream_k, self.stream_v = [None] * L, [None] * L
        self.n_ret = [int((self.labels[i] >= 0.5).sum()) for i in range(L)]  # :264-266
        self.n_str = [self.labels.shape[1] - n for n in self.n_ret]

    def append_layer(self, layer_idx: int, k, v):
        """benchmark_llama31.py:171-184 (k/v in reordered head order, (B,G,S,D))."""
        nr = self.n_ret[layer_idx]
        if nr > 0:
            rk, rv = k[:, :nr], v[:, :nr]
            if self.full_k[layer_idx] is None:
                self.full_k[layer_idx], self.full_v[layer_idx] = rk.copy(), rv.copy()
            else:
                self.full_k[layer_idx] = np.concatenate([self.full_k[layer_idx], rk], axis=2)
                self.full_v[layer_idx] = np.concatenate([self.full_v[layer_idx], rv], axis=2)
        if self.n_str[layer_idx] > 0:
            sk, sv = k[:, nr:], v[:, nr:]
            if self.stream_k[layer_idx] is not None:
                sk = np.concatenate([self.stream_k[layer_idx], sk], axis=2)
                sv = np.concatenate([self.stream_v[layer_idx], sv], axis=2)
            self.stream_k[layer_idx], self.stream_v[layer_idx] = compress_stream(
                sk, sv, self.sink_size, self.recent_size)


def layer_attention(cache: OracleKVCache, layer_idx: int, q, k, v) -> np.ndarray:
    """One layer of the patched attention forward, from post-RoPE q/k/v to the
    attention output in ORIGINAL head order; benchmark_llama31.py:187-253
    (the projections, RoPE and o_proj are outside this boundary).

    q (B,C,Hq,D), k/v (B,C,G,D) float32 (bf16 values when cache.dtype == 'bf16')
    -> (B,C,Hq,D).  Appends k/v to the cache; advances kv_seq_len after the
    last layer (benchmark_llama31.py:248-250)."""
    B, C, Hq, D = q.shape
    G = k.shape[2]
    grp = Hq // G
    if cache.backend == "flash":
        return _layer_attention_flash(cache, layer_idx, q, k, v)
    kv_perm, q_perm = head_permutation(cache.labels[layer_idx], Hq, G)
    qh = np.ascontiguousarray(np.transpose(q, (0, 2, 1, 3))[:, q_perm])   # (B,Hq,C,D)
    kh = np.ascontiguousarray(np.transpose(k, (0, 2, 1, 3))[:, kv_perm])  # (B,G,C,D)
    vh = np.ascontiguousarray(np.transpose(v, (0, 2, 1, 3))[:, kv_perm])
    nr, ns = cache.n_ret[layer_idx], cache.n_str[layer_idx]
    past_len = cache.kv_seq_len
    outs = []
    if nr > 0:
        ofk, ofv = cache.full_k[layer_idx], cache.full_v[layer_idx]
        fk = kh[:, :nr] if ofk is None else np.concatenate([ofk, kh[:, :nr]], axis=2)
        fv = vh[:, :nr] if ofv is None else np.concatenate([ofv, vh[:, :nr]], axis=2)
        outs.append(eager_attention(qh[:, : nr * grp], repeat_kv(fk, grp), repeat_kv(fv, grp),
                                    past_len, causal=(C > 1), dtype=cache.dtype))
    if ns > 0:
        osk, osv = cache.stream_k[layer_idx], cache.stream_v[layer_idx]
        sk = kh[:, nr:] if osk is None else np.concatenate([osk, kh[:, nr:]], axis=2)
        sv = vh[:, nr:] if osv is None else np.concatenate([osv, vh[:, nr:]], axis=2)
        outs.append(streaming_attention(
            qh[:, nr * grp:], repeat_kv(sk, grp), repeat_kv(sv, grp), past_len=past_len,
            cached_len=0 if osk is None else osk.shape[2], sink_size=cache.sink_size,
            recent_size=cache.recent_size, dtype=cache.dtype))
    out_perm = np.concatenate(outs, axis=1) if len(outs) > 1 else outs[0]   # (B,Hq,C,D)
    out = np.empty_like(out_perm)
    out[:, q_perm] = out_perm
    cache.append_layer(layer_idx, kh, vh)
    if layer_idx == cache.num_layers - 1:
        cache.kv_seq_len += C
    return np.ascontiguousarray(np.transpose(out, (0, 2, 1, 3)))


def _layer_attention_flash(cache: OracleKVCache, layer_idx: int, q, k, v) -> np.ndarray:
    """The layer's attention under the decoding-simulation protocol;
    eval/efficiency/attention_utils.py:45-89 (aoh_flash_attention, driven by
    make_aoh_forward's flash branch, benchmark_llama31.py:212-215):

    * the first call of a layer (its cache empty): every head, streaming heads
      too, attends causally to the whole chunk (flash_attn_func causal over all
      heads, :62-67);
    * later calls: retrieval heads attend to their cached keys and the chunk,
      streaming heads to their kept keys (sink + recent) and the chunk, both
      causal with the queries aligned to the end of the keys (flash-attn's
      causal convention when there are more keys than queries, :69-80) -- no
      window mask;
    * then the cache keeps every retrieval row and the sink and recent rows of
      each streaming head (the in-place trim of :82-86 keeps exactly what
      compress_stream keeps).

    The arithmetic is the eager restatement's (fp32 scores and softmax,
    probabilities rounded to the dtype); flash-attn's own rounding of the
    unnormalised probabilities differs from it by at most a few ulps."""
    B, C, Hq, D = q.shape
    G = k.shape[2]
    grp = Hq // G
    kv_perm, q_perm = head_permutation(cache.labels[layer_idx], Hq, G)
    qh = np.ascontiguousarray(np.transpose(q, (0, 2, 1, 3))[:, q_perm])
    kh = np.ascontiguousarray(np.transpose(k, (0, 2, 1, 3))[:, kv_perm])
    vh = np.ascontiguousarray(np.transpose(v, (0, 2, 1, 3))[:, kv_perm])
    nr, ns = cache.n_ret[layer_idx], cache.n_str[layer_idx]
    prefill = cache.full_k[layer_idx] is None and cache.stream_k[layer_idx] is None
    if prefill:
        out_perm = eager_attention(qh, repeat_kv(kh, grp), repeat_kv(vh, grp), 0, causal=True, dtype=cache.dtype)
    else:
        outs = []
        if nr > 0:
            fk = np.concatenate([cache.full_k[layer_idx], kh[:, :nr]], axis=2)
            fv = np.concatenate([cache.full_v[layer_idx], vh[:, :nr]], axis=2)
            outs.append(eager_attention(qh[:, : nr * grp], repeat_kv(fk, grp), repeat_kv(fv, grp),
                                        fk.shape[2] - C, causal=True, dtype=cache.dtype))
        if ns > 0:
            sk = np.concatenate([cache.stream_k[layer_idx], kh[:, nr:]], axis=2)
            sv = np.concatenate([cache.stream_v[layer_idx], vh[:, nr:]], axis=2)
            outs.append(eager_attention(qh[:, nr * grp:], repeat_kv(sk, grp), repeat_kv(sv, grp),
                                        sk.shape[2] - C, causal=True, dtype=cache.dtype))
        out_perm = np.concatenate(outs, axis=1) if len(outs) > 1 else outs[0]
    out = np.empty_like(out_perm)
    out[:, q_perm] = out_perm
    cache.append_layer(layer_idx, kh, vh)
    if layer_idx == cache.num_layers - 1:
        cache.kv_seq_len += C
    return np.ascontiguousarray(np.transpose(out, (0, 2, 1, 3)))


def decode_from_state(q, k_new, v_new, k_ctx, v_ctx, labels_row, past_len: int,
                      sink_size: int, recent_size: int, dtype: str) -> np.ndarray:
    """Decode step (q_len = 1) of one layer over an already-filled context.

    ``k_ctx``/``v_ctx`` (B,T,G,D) hold the full history of every KV head (the
    state a prefill leaves behind, before trimming); streaming heads see only
    ``compress_stream`` of it, exactly what AoHKVCache keeps
    (benchmark_llama31.py:171-184).  Same arithmetic as :func:`layer_attention`
    with a single query token."""
    B, _, Hq, D = q.shape
    G = k_new.shape[2]
    grp = Hq // G
    out = np.empty((B, 1, Hq, D), dtype=F32)
    T = past_len
    for g in range(G):
        qg = np.transpose(q[:, :, g * grp:(g + 1) * grp], (0, 2, 1, 3))        # (B,grp,1,D)
        kc = np.transpose(k_ctx[:, :T, g:g + 1], (0, 2, 1, 3))                  # (B,1,T,D)
        vc = np.transpose(v_ctx[:, :T, g:g + 1], (0, 2, 1, 3))
        kn = np.transpose(k_new[:, :, g:g + 1], (0, 2, 1, 3))
        vn = np.transpose(v_new[:, :, g:g + 1], (0, 2, 1, 3))
        if labels_row[g] >= 0.5:
            kk = np.concatenate([kc, kn], axis=2)
            vv = np.concatenate([vc, vn], axis=2)
            o = eager_attention(qg, repeat_kv(kk, grp), repeat_kv(vv, grp), T, False, dtype)
        else:
            ks, vs = compress_stream(kc, vc, sink_size, recent_size)
            kk = np.concatenate([ks, kn], axis=2)
            vv = np.concatenate([vs, vn], axis=2)
            o = streaming_attention(qg, repeat_kv(kk, grp), repeat_kv(vv, grp), past_len=T,
                                    cached_len=ks.shape[2], sink_size=sink_size,
                                    recent_size=recent_size, dtype=dtype)
        out[:, :, g * grp:(g + 1) * grp] = np.transpose(o, (0, 2, 1, 3))
    return out


def attend_rows(q_rows, q_pos, k_hist, v_hist, retrieval: bool, sink_size: int, recent_size: int,
                dtype: str, block: int = 32) -> np.ndarray:
    """Chosen query rows of one KV group over its full key history, for checks
    at full context sizes where running every row is too slow.

    ``q_rows`` (R, grp, D) at positions ``q_pos`` (R,); ``k_hist``/``v_hist``
    (S, D) hold positions 0..S-1 of the group's keys (cached ones and this
    chunk's).  A retrieval row at position p sees keys 0..p (the causal mask
    offset by past_len, benchmark_llama31.py:116-120 and :123-132); a streaming
    row sees keys k <= p with k < sink or k >= p - recent
    (attention_utils.py:109-114), which are exactly the keys the reference's
    compressed cache plus the chunk still hold for it (compress_stream keeps the
    last ``recent`` cached positions, :23-42).  Same arithmetic as the
    reference: fp32 scores times D^-0.5, masked scores finfo(float32).min,
    fp32 softmax, probabilities rounded to the input dtype, fp32 P.V rounded to
    the input dtype.  GQA expansion (repeat_kv) only copies, so the group's
    query heads are evaluated against the one KV head directly.
    -> (R, grp, D) float32."""
    q_rows = np.asarray(q_rows, dtype=F32)
    R, grp, D = q_rows.shape
    scale = F32(D ** -0.5)
    kf = np.asarray(k_hist, dtype=F32)
    vf = np.asarray(v_hist, dtype=F32)
    kpos = np.arange(kf.shape[0])
    out = np.empty((R, grp, D), dtype=F32)
    for r0 in range(0, R, block):
        r1 = min(R, r0 + block)
        p = np.asarray(q_pos[r0:r1])[:, None]
        hi = int(p.max()) + 1
        allowed = kpos[None, :hi] <= p
        if not retrieval:
            allowed &= (kpos[None, :hi] < sink_size) | (kpos[None, :hi] >= p - recent_size)
        scores = np.matmul(q_rows[r0:r1], kf[:hi].T) * scale                 # (r, grp, hi)
        scores = np.where(allowed[:, None, :], scores, _NEG).astype(F32)
        out[r0:r1] = _pv(_softmax_f32(scores), vf[:hi], dtype)
    return out


def decode_unit(q_grp, k_new, v_new, k_cached, v_cached, retrieval: bool, past_len: int,
                sink_size: int, recent_size: int, dtype: str) -> np.ndarray:
    """Decode step (q_len = 1) of one (sequence, KV head) unit: what
    :func:`layer_attention` computes for that unit, from the unit's cached rows
    as AoHKVCache holds them (retrieval: all ``past_len`` rows; streaming:
    ``compress_stream`` of the history, sink then recent rows).
    ``q_grp`` (grp, D), ``k_new``/``v_new`` (D,), ``k_cached``/``v_cached``
    (S, D).  Retrieval: eager_attention without a mask (q_len = 1,
    benchmark_llama31.py:123-132); streaming: streaming_attention
    (attention_utils.py:92-119).  GQA expansion (repeat_kv) only copies, so the
    group's query heads are evaluated against the one KV head directly.
    -> (grp, D) float32."""
    q = np.asarray(q_grp, dtype=F32)[None, :, None, :]                        # (1, grp, 1, D)
    kk = np.concatenate([np.asarray(k_cached, dtype=F32), np.asarray(k_new, dtype=F32)[None]], 0)[None, None]
    vv = np.concatenate([np.asarray(v_cached, dtype=F32), np.asarray(v_new, dtype=F32)[None]], 0)[None, None]
    if retrieval:
        o = eager_attention(q, kk, vv, past_len, False, dtype)
    else:
        o = streaming_attention(q, kk, vv, past_len=past_len, cached_len=kk.shape[2] - 1,
                                sink_size=sink_size, recent_size=recent_size, dtype=dtype)
    return o[0, :, 0]


# ----------------------------------------------------------------------------
# effective-rank classifier
# ----------------------------------------------------------------------------

def gram_matrix(wq_h: np.ndarray, wk_g: np.ndarray, binary: bool, exact: bool = False) -> np.ndarray:
    """C = (W_Q W_Q^T)(W_K W_K^T); aoh/effective_rank.py:27-42, binary :45-59.

    ``exact=False`` computes in float32 like the reference; ``exact=True``
    computes in float64 (integers are exact there in binary mode)."""
    dt = np.float64 if exact else F32
    a = wq_h.astype(dt)
    b = wk_g.astype(dt)
    if binary:
        a, b = np.sign(a), np.sign(b)
    qq = a @ a.T
    kk = b @ b.T
    return qq @ kk


def eigenvalues_to_eff_rank(eigs: np.ndarray, exact: bool = False) -> float:
    """sigma = sqrt(|lambda|+eps), p = sigma/sum, H = -sum p log(p+eps), exp(H);
    aoh/effective_rank.py:62-85 (float32 arithmetic unless ``exact``)."""
    dt = np.float64 if exact else F32
    sigma = np.sqrt(np.abs(eigs).astype(dt) + dt(EPS))
    s = sigma.sum(dtype=dt)
    if s < EPS:
        return 1.0
    p = sigma / s
    h = -(p * np.log(p + dt(EPS))).sum(dtype=dt)
    return float(np.exp(h))


def compute_eff_rank(wq_h, wk_g, binary: bool = False, exact: bool = False) -> float:
    """aoh/effective_rank.py:88-106 (eigvals of the non-symmetric C)."""
    c = gram_matrix(wq_h, wk_g, binary, exact)
    if exact:
        # C = QQ.KK with QQ, KK symmetric positive semi-definite: its eigenvalues
        # are those of the symmetric L^T KK L (QQ = L L^T), solved in float64.
        a = wq_h.astype(np.float64)
        b = wk_g.astype(np.float64)
        if binary:
            a, b = np.sign(a), np.sign(b)
        qq, kk = a @ a.T, b @ b.T
        lq = np.linalg.cholesky(qq)
        eigs = np.linalg.eigvalsh(lq.T @ kk @ lq)
    else:
        eigs = np.linalg.eigvals(c)
    return eigenvalues_to_eff_rank(eigs, exact)


def compute_all_eff_ranks(wq_layers, wk_layers, num_q: int, num_kv: int, head_dim: int,
                          binary: bool = False, exact: bool = False) -> np.ndarray:
    """(L, H) float64; aoh/effective_rank.py:109-142.  ``wq_layers[l]`` is the
    layer's q_proj.weight (H*D, d_model), ``wk_layers[l]`` its k_proj.weight."""
    L = len(wq_layers)
    grp = num_q // num_kv
    out = np.zeros((L, num_q), dtype=np.float64)
    for l in range(L):
        wq = np.asarray(wq_layers[l], dtype=F32).reshape(num_q, head_dim, -1)  # weight_extract.py:104-111
        wk = np.asarray(wk_layers[l], dtype=F32).reshape(num_kv, head_dim, -1)
        for h in range(num_q):
            r = compute_eff_rank(wq[h], wk[h // grp], binary, exact)
            out[l, h] = float(np.float32(r))  # the reference stores float(fp32 .item())
    return out


def aggregate_kv(eff_ranks_q: np.ndarray, num_kv: int, agg: str) -> np.ndarray:
    """GQA aggregation in float64; aoh/classifier.py:102-116."""
    if agg not in ("mean", "min", "max"):  # classifier.py:41-42
        raise ValueError(f"agg must be 'mean', 'min', or 'max', got {agg!r}")
    L, H = eff_ranks_q.shape
    if num_kv == H:
        return eff_ranks_q.copy()
    grp = H // num_kv
    out = np.zeros((L, num_kv), dtype=np.float64)
    for l in range(L):
        for g in range(num_kv):
            r = eff_ranks_q[l, g * grp:(g + 1) * grp]
            out[l, g] = r.mean() if agg == "mean" else (r.min() if agg == "min" else r.max())
    return out


def classify_labels(eff_ranks_kv: np.ndarray, sparsity: float) -> np.ndarray:
    """Lowest-rank k KV heads per layer are retrieval; aoh/classifier.py:118-128."""
    L, G = eff_ranks_kv.shape
    k = max(0, min(G, round((1.0 - sparsity) * G)))
    labels = np.zeros((L, G), dtype=np.float64)
    for l in range(L):
        labels[l, np.argsort(eff_ranks_kv[l])[:k]] = 1.0
    return labels


def kv_storage_gb_aoh(num_layers, head_dim, n_ret, n_str, total_len, sink_size, recent_size,
                      dtype_bytes: int = 2) -> float:
    """Analytical KV storage; eval/efficiency/benchmark_llama31.py:345-351."""
    stream_len = min(total_len, sink_size + recent_size)
    elems = 0
    for nr, ns in zip(n_ret, n_str):
        elems += 2 * (nr * total_len + ns * stream_len) * head_dim
    return elems * dtype_bytes / 1e9


def attention_flops(q_len: int, past_len: int, retrieval: bool, sink: int, recent: int,
                    head_dim: int = 128) -> int:
    """Masked-in (query, key) pairs x 4*D for one query head over one chunk."""
    qp = np.arange(past_len, past_len + q_len, dtype=np.int64)
    if retrieval:
        pairs = (qp + 1).sum()
    else:
        pairs = (np.minimum(qp + 1, sink) + np.maximum(0, qp + 1 - np.maximum(sink, qp - recent))).sum()
    return int(pairs) * 4 * head_dim
