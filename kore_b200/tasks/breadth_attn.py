"""Breadth families, part 5: attention variants beyond plain causal / sliding.

Every variant is a module-level PyTorch definition on (B, H, Sq, D) queries and
(B, KV, S, D) keys / values (GQA / MQA by ``KV < H``) that serves as the fp32
oracle, the vendor baseline in the task dtype (SDPA with an additive mask where
the variant is expressible that way, else the same definition) and the seed:

* positional biases: ALiBi (prefill and decode), T5 bucketed relative bias,
  learned attention sinks;
* masks: arbitrary boolean mask, dilated causal, chunked (block-local) causal,
  prefix-LM (bidirectional prefix, causal tail), windows of 256 / 1024;
* layouts: cross attention (prefill and single step), packed variable-length
  sequences (``cu_seqlens``, causal and full), KV-cache append then decode,
  paged decode through a block table, decode at head dims 64 / 128 / 256;
* numerics: fp8 (e4m3, per-tensor scales) prefill, q/k RMS-normalised
  attention, sigmoid attention (no softmax), soft-capped decode;
* training: the attention backward (dQ, dK, dV from dO).

Reference parity: task dirs ``genb_attn2_*`` / ``genb_attn_*`` of the
reference (kore/tasks/breadth/attn2_ext.py, attn_ext.py), written from the
operator definitions, not from that code.
"""
from __future__ import annotations

import math
from typing import Callable, Dict, List

import torch
import torch.nn.functional as F

from .spec import OpSpec, _gen, _randn

FP8_MAX = 448.0


def _fp32_of(f):
    return lambda *x: f(*(t.float() if t.is_floating_point() else t for t in x))


def _seed_for(entry: str, args: str, fn: Callable) -> str:
    return (f"from kore_b200.tasks.breadth_attn import {fn.__name__} as _ref\n\n\n"
            f"def {entry}({args}):\n    return _ref({args})\n")


def _expand(q, k, v):
    H, KV = q.shape[1], k.shape[1]
    if H != KV:
        k = k.repeat_interleave(H // KV, 1)
        v = v.repeat_interleave(H // KV, 1)
    return k, v


def _softmax_attend(q, k, v, bias=None, mask=None):
    """softmax(q k^T / sqrt(D) + bias, masked) v with fp32 scores."""
    k, v = _expand(q, k, v)
    sc = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    if bias is not None:
        sc = sc + bias.float()
    if mask is not None:
        sc = sc.masked_fill(mask, float("-inf"))
    p = torch.softmax(sc, -1).nan_to_num(0.0)
    return (p @ v.float()).to(q.dtype)


def _pos(Sq, S, dev):
    qi = torch.arange(Sq, device=dev)[:, None] + (S - Sq)
    ki = torch.arange(S, device=dev)[None, :]
    return qi, ki


# ============================================================================= inputs
def mk_qkv(d, s, dev, dt):
    B, H, KV, S, D = d["B"], d["H"], d["KV"], d["S"], d["D"]
    Sq = d.get("Sq", S)
    return (_randn((B, H, Sq, D), s, dev, dt), _randn((B, KV, S, D), s + 1, dev, dt),
            _randn((B, KV, S, D), s + 2, dev, dt))


def mk_qkv_mask(d, s, dev, dt):
    q, k, v = mk_qkv(d, s, dev, dt)
    Sq, S = q.shape[2], k.shape[2]
    g = _gen(s + 3, dev)
    m = torch.rand((Sq, S), generator=g, device=dev) < 0.3
    m[:, 0] = False                    # every row keeps at least one key
    return q, k, v, m


def mk_qkv_t5(d, s, dev, dt):
    q, k, v = mk_qkv(d, s, dev, dt)
    table = _randn((32, q.shape[1]), s + 3, dev, torch.float32, 0.5).to(dt)
    return q, k, v, table


def mk_qkv_sink(d, s, dev, dt):
    q, k, v = mk_qkv(d, s, dev, dt)
    return q, k, v, _randn((q.shape[1],), s + 3, dev, torch.float32).to(dt)


def mk_varlen(d, s, dev, dt):
    """Packed (T, H, D) queries and (T, KV, D) keys/values of ``n`` sequences
    of deterministic ragged lengths summing to S."""
    H, KV, S, D, n = d["H"], d["KV"], d["S"], d["D"], d.get("nseq", 4)
    g = torch.Generator().manual_seed(int(s) + 11)
    cuts = sorted(torch.randperm(S - 1, generator=g)[: n - 1].add(1).tolist())
    cu = torch.tensor([0] + cuts + [S], dtype=torch.int32, device=dev)
    return (_randn((S, H, D), s, dev, dt), _randn((S, KV, D), s + 1, dev, dt), _randn((S, KV, D), s + 2, dev, dt), cu)


def mk_cache_append(d, s, dev, dt):
    """One decode step: new K/V rows are written at position ``pos`` of a
    (B, KV, Smax, D) cache, then the query attends to positions 0..pos."""
    B, H, KV, S, D = d["B"], d["H"], d["KV"], d["S"], d["D"]
    kc = _randn((B, KV, S, D), s + 1, dev, dt)
    vc = _randn((B, KV, S, D), s + 2, dev, dt)
    kn = _randn((B, KV, 1, D), s + 3, dev, dt)
    vn = _randn((B, KV, 1, D), s + 4, dev, dt)
    pos = torch.tensor([S * 3 // 4], dtype=torch.int64, device=dev)
    return _randn((B, H, 1, D), s, dev, dt), kc, vc, kn, vn, pos


def mk_paged(d, s, dev, dt):
    """Decode through a block table: K/V pages of 16 tokens in a shuffled pool."""
    B, H, KV, S, D = d["B"], d["H"], d["KV"], d["S"], d["D"]
    P = 16
    nb = S // P
    pool = B * nb
    g = torch.Generator().manual_seed(int(s) + 5)
    table = torch.randperm(pool, generator=g).view(B, nb).to(device=dev, dtype=torch.int32)
    kp = _randn((pool, KV, P, D), s + 1, dev, dt)
    vp = _randn((pool, KV, P, D), s + 2, dev, dt)
    return _randn((B, H, 1, D), s, dev, dt), kp, vp, table


def mk_bwd(d, s, dev, dt):
    q, k, v = mk_qkv(d, s, dev, dt)
    return q, k, v, _randn(q.shape, s + 3, dev, dt)


# ============================================================================= definitions
def alibi_slopes(H: int, dev) -> torch.Tensor:
    """Geometric ALiBi slopes 2^(-8 i / n) for the nearest power of two n >= H,
    interleaved for the remainder (Press et al., 2022)."""
    n = 2 ** math.ceil(math.log2(H))
    base = torch.tensor([2.0 ** (-8.0 * (i + 1) / n) for i in range(n)], device=dev)
    if n == H:
        return base
    return torch.cat([base[0::2], base[1::2]])[:H]


def attn_alibi_causal(q, k, v):
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    bias = -alibi_slopes(q.shape[1], q.device)[:, None, None] * (qi - ki).clamp(min=0).float()
    return _softmax_attend(q, k, v, bias=bias, mask=ki > qi)


def t5_bucket(rel: torch.Tensor, buckets: int = 32, max_distance: int = 128) -> torch.Tensor:
    """Causal T5 relative-position buckets: exact for distances < buckets/2,
    logarithmic up to ``max_distance`` beyond (Raffel et al., 2020)."""
    n = (-rel).clamp(min=0)
    exact = buckets // 2
    big = exact + (torch.log(n.float().clamp(min=1) / exact) / math.log(max_distance / exact)
                   * (buckets - exact)).long()
    return torch.where(n < exact, n, big.clamp(max=buckets - 1))


def attn_relbias_t5_causal(q, k, v, table):
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    b = t5_bucket(ki - qi, table.shape[0])
    bias = table.float()[b].permute(2, 0, 1)               # (H, Sq, S)
    return _softmax_attend(q, k, v, bias=bias, mask=ki > qi)


def attn_custom_mask(q, k, v, mask):
    return _softmax_attend(q, k, v, mask=mask.bool())


def attn_dilated_causal(q, k, v):
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    return _softmax_attend(q, k, v, mask=(ki > qi) | ((qi - ki) % 2 != 0))


def attn_chunked_causal(q, k, v):
    """Block-local causal attention: a query sees earlier keys of its own
    512-token chunk only."""
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    return _softmax_attend(q, k, v, mask=(ki > qi) | (ki // 512 != qi // 512))


def attn_prefix_lm(q, k, v):
    """The first quarter of the sequence attends bidirectionally, the rest causally."""
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    pre = S // 4
    return _softmax_attend(q, k, v, mask=(ki > qi) & (ki >= pre))


def attn_window256(q, k, v):
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    return _softmax_attend(q, k, v, mask=(ki > qi) | (ki <= qi - 256))


def attn_window1024(q, k, v):
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    return _softmax_attend(q, k, v, mask=(ki > qi) | (ki <= qi - 1024))


def attn_cross(q, k, v):
    return _softmax_attend(q, k, v)


def attn_sink_causal(q, k, v, sink):
    """Causal attention with one learned per-head sink logit in the softmax
    denominator (it takes probability mass but contributes no value)."""
    k2, v2 = _expand(q, k, v)
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    sc = (q.float() @ k2.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    sc = sc.masked_fill(ki > qi, float("-inf"))
    col = sink.float()[None, :, None, None].expand(q.shape[0], -1, Sq, 1)
    p = torch.softmax(torch.cat([sc, col], -1), -1)[..., :-1]
    return (p @ v2.float()).to(q.dtype)


def attn_varlen_causal(q, k, v, cu):
    return _varlen(q, k, v, cu, True)


def attn_varlen_full(q, k, v, cu):
    return _varlen(q, k, v, cu, False)


def _varlen(q, k, v, cu, causal):
    out = torch.empty_like(q)
    c = cu.tolist()
    for a, b in zip(c[:-1], c[1:]):
        qs, ks, vs = (t[a:b].transpose(0, 1)[None] for t in (q, k, v))
        m = None
        if causal:
            qi, ki = _pos(b - a, b - a, q.device)
            m = ki > qi
        out[a:b] = _softmax_attend(qs, ks, vs, mask=m)[0].transpose(0, 1)
    return out


def attn_cache_append_decode(q, kc, vc, kn, vn, pos):
    p = int(pos.reshape(-1)[0])
    k = kc.clone()
    v = vc.clone()
    k[:, :, p] = kn[:, :, 0]
    v[:, :, p] = vn[:, :, 0]
    return _softmax_attend(q, k[:, :, : p + 1], v[:, :, : p + 1])


def attn_paged_decode(q, kp, vp, table):
    B = q.shape[0]
    KV, P, D = kp.shape[1], kp.shape[2], kp.shape[3]
    k = kp[table.long()].permute(0, 2, 1, 3, 4).reshape(B, KV, -1, D)
    v = vp[table.long()].permute(0, 2, 1, 3, 4).reshape(B, KV, -1, D)
    return _softmax_attend(q, k, v)


def attn_decode(q, k, v):
    return _softmax_attend(q, k, v)


def attn_alibi_decode(q, k, v):
    S = k.shape[2]
    dist = (S - 1 - torch.arange(S, device=q.device)).float()
    bias = -alibi_slopes(q.shape[1], q.device)[:, None, None] * dist
    return _softmax_attend(q, k, v, bias=bias)


def attn_softcap_decode(q, k, v):
    k2, v2 = _expand(q, k, v)
    sc = (q.float() @ k2.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    sc = 50.0 * torch.tanh(sc / 50.0)
    return (torch.softmax(sc, -1) @ v2.float()).to(q.dtype)


def _fp8_roundtrip(x):
    s = x.float().abs().amax().clamp(min=1e-12) / FP8_MAX
    return (x.float() / s).clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).float() * s


def attn_fp8_causal(q, k, v):
    """q, k, v quantised to e4m3 with per-tensor scales, attention in fp32
    scores, output in the input dtype."""
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    out = _softmax_attend(_fp8_roundtrip(q), _fp8_roundtrip(k), _fp8_roundtrip(v), mask=ki > qi)
    return out.to(q.dtype)


def attn_fp8_full(q, k, v):
    return _softmax_attend(_fp8_roundtrip(q), _fp8_roundtrip(k), _fp8_roundtrip(v)).to(q.dtype)


def attn_qknorm_causal(q, k, v):
    """Qwen3-style attention: q and k RMS-normalised over the head dim first."""
    def rms(x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype)
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    return _softmax_attend(rms(q), rms(k), v, mask=ki > qi)


def attn_sigmoid_causal(q, k, v):
    """Sigmoid attention: sigmoid(q k^T / sqrt(D) - log S) instead of softmax."""
    k2, v2 = _expand(q, k, v)
    Sq, S = q.shape[2], k.shape[2]
    qi, ki = _pos(Sq, S, q.device)
    sc = (q.float() @ k2.float().transpose(-1, -2)) / math.sqrt(q.shape[-1]) - math.log(S)
    p = torch.sigmoid(sc).masked_fill(ki > qi, 0.0)
    return (p @ v2.float()).to(q.dtype)


def attn_bwd_causal(q, k, v, do):
    """dQ, dK and dV of causal softmax attention for upstream gradient ``do``,
    each flattened and concatenated into one vector in the input dtype."""
    with torch.enable_grad():
        qf, kf, vf = (t.detach().float().requires_grad_(True) for t in (q, k, v))
        Sq, S = q.shape[2], k.shape[2]
        qi, ki = _pos(Sq, S, q.device)
        k2, v2 = _expand(qf, kf, vf)
        sc = (qf @ k2.transpose(-1, -2)) / math.sqrt(q.shape[-1])
        o = torch.softmax(sc.masked_fill(ki > qi, float("-inf")), -1) @ v2
        dq, dk, dv = torch.autograd.grad(o, (qf, kf, vf), do.float())
    return torch.cat([dq.flatten(), dk.flatten(), dv.flatten()]).to(q.dtype)


# ---------------------------------------------------------------- vendor baselines
def _sdpa_mask(fn_mask):
    def f(q, k, v, *extra):
        with torch.no_grad():
            return F.scaled_dot_product_attention(q, k, v, attn_mask=fn_mask(q, k, *extra), enable_gqa=True)
    return f


def _alibi_bias(q, k):
    qi, ki = _pos(q.shape[2], k.shape[2], q.device)
    bias = -alibi_slopes(q.shape[1], q.device)[:, None, None] * (qi - ki).clamp(min=0).float()
    return bias.masked_fill(ki > qi, float("-inf")).to(q.dtype)


def _window_mask(w):
    def m(q, k):
        qi, ki = _pos(q.shape[2], k.shape[2], q.device)
        return ~((ki > qi) | (ki <= qi - w))
    return m


def _plain_baseline(fn):
    def f(*x):
        with torch.no_grad():
            return fn(*x)
    return f


# ============================================================================= table
_LAYOUTS = {"mha": (16, 16), "gqa": (32, 8), "mqa": (32, 1)}


def _dims(layout: str, **kw) -> Dict[str, int]:
    h, kv = _LAYOUTS[layout]
    d = {"B": 2, "H": h, "KV": kv, "S": 2048, "D": 128}
    d.update(kw)
    return d


def _mini(d: Dict[str, int]) -> Dict[str, int]:
    m = dict(d, B=1, H=max(2, d["H"] // 8), KV=max(1, d["KV"] // 8))
    if m["H"] % m["KV"]:
        m["KV"] = 1
    m["S"] = min(d["S"], 96 if "nseq" not in d else 64)
    if "Sq" in d:
        m["Sq"] = 1 if d["Sq"] == 1 else min(d["Sq"], 48)
    m["D"] = min(d["D"], 64)
    return m


Entry = tuple  # (name, operation, entry, make, fn, args, dims, baseline or None)


def _table() -> List[Entry]:
    T: List[Entry] = []
    for lay in ("mha", "gqa", "mqa"):
        T.append((f"alibi_{lay}_causal", "attention", mk_qkv, attn_alibi_causal, "q, k, v", _dims(lay),
                  _sdpa_mask(_alibi_bias)))
        T.append((f"chunked_{lay}_causal", "attention", mk_qkv, attn_chunked_causal, "q, k, v", _dims(lay), None))
        T.append((f"cacheappend_{lay}", "attention_decode", mk_cache_append, attn_cache_append_decode,
                  "q, kc, vc, kn, vn, pos", _dims(lay, B=16, S=4096), None))
        T.append((f"alibi_decode_{lay}", "attention_decode", mk_qkv, attn_alibi_decode, "q, k, v",
                  _dims(lay, B=16, S=4096, Sq=1), None))
    for lay in ("mha", "gqa"):
        T.append((f"relbias_t5_{lay}_causal", "attention", mk_qkv_t5, attn_relbias_t5_causal, "q, k, v, table",
                  _dims(lay), None))
        T.append((f"custommask_{lay}", "attention", mk_qkv_mask, attn_custom_mask, "q, k, v, mask", _dims(lay),
                  _sdpa_mask(lambda q, k, m: ~m.bool())))
        T.append((f"dilated_{lay}_causal", "attention", mk_qkv, attn_dilated_causal, "q, k, v", _dims(lay), None))
        T.append((f"prefixlm_{lay}", "attention", mk_qkv, attn_prefix_lm, "q, k, v", _dims(lay), None))
        T.append((f"cross_{lay}_prefill", "attention", mk_qkv, attn_cross, "q, k, v", _dims(lay, Sq=1024, S=4096),
                  _sdpa_mask(lambda q, k: None)))
        T.append((f"cross_{lay}_step", "attention_decode", mk_qkv, attn_cross, "q, k, v",
                  _dims(lay, B=32, Sq=1, S=1500), _sdpa_mask(lambda q, k: None)))
        T.append((f"sink_{lay}_causal", "attention", mk_qkv_sink, attn_sink_causal, "q, k, v, sink", _dims(lay), None))
        T.append((f"sigmoid_{lay}_causal", "attention", mk_qkv, attn_sigmoid_causal, "q, k, v", _dims(lay), None))
        for w, fn in ((256, attn_window256), (1024, attn_window1024)):
            T.append((f"window{w}_{lay}_causal", "attention", mk_qkv, fn, "q, k, v", _dims(lay, S=4096),
                      _sdpa_mask(_window_mask(w))))
        for c, fn in (("causal", attn_varlen_causal), ("noncausal", attn_varlen_full)):
            T.append((f"varlen_{lay}_{c}", "attention", mk_varlen, fn, "q, k, v, cu",
                      _dims(lay, B=1, S=8192, nseq=6), None))
    for lay in ("gqa", "mqa"):
        for hd in (64, 128, 256):
            T.append((f"decode_{lay}_hd{hd}", "attention_decode", mk_qkv, attn_decode, "q, k, v",
                      _dims(lay, B=32, S=4096, Sq=1, D=hd), _sdpa_mask(lambda q, k: None)))
        T.append((f"paged_decode_{lay}", "attention_decode", mk_paged, attn_paged_decode, "q, kp, vp, table",
                  _dims(lay, B=32, S=4096), None))
        T.append((f"softcap_decode_{lay}", "attention_decode", mk_qkv, attn_softcap_decode, "q, k, v",
                  _dims(lay, B=32, S=4096, Sq=1), None))
        T.append((f"qknorm_{lay}_causal", "attention", mk_qkv, attn_qknorm_causal, "q, k, v", _dims(lay), None))
    for lay in ("mha", "gqa", "mqa"):
        T.append((f"bwd_{lay}_causal", "attention_backward", mk_bwd, attn_bwd_causal, "q, k, v, do",
                  _dims(lay, S=1024), None))
    return T


_FP8 = [("fp8_gqa_prefill_causal", attn_fp8_causal, "gqa"), ("fp8_gqa_prefill_noncausal", attn_fp8_full, "gqa"),
        ("fp8_mqa_prefill_causal", attn_fp8_causal, "mqa"), ("fp8_mha_prefill_causal", attn_fp8_causal, "mha")]


def build() -> List[OpSpec]:
    out: List[OpSpec] = []
    for dt in ("bf16", "fp16"):
        for name, op, mk, fn, args, d, base in _table():
            out.append(OpSpec(f"genb_attn2_{name}_{dt}", op, "attention", mk, _fp32_of(fn),
                              base or _plain_baseline(fn), _seed_for("attention", args, fn),
                              {"minimal": _mini(d), "primary": d, "validation": []}, "attention_ext", dt))
    for name, fn, lay in _FP8:
        d = _dims(lay)
        out.append(OpSpec(f"genb_attn2_{name}_fp8", "attention", "attention", mk_qkv, _fp32_of(fn),
                          _plain_baseline(fn), _seed_for("attention", "q, k, v", fn),
                          {"minimal": _mini(d), "primary": d, "validation": []}, "attention_ext", "fp8"))
    return out
