"""Hand-authored core task families and the ``genv_*`` vendor-op tasks.

Every task here is one PyTorch source (the seed the policy starts from) that
defines the entry point; the same source run on fp32 copies of the inputs is
the oracle, and the vendor baseline on B200 is a library kernel where one
exists (cuBLAS through ``torch.matmul``, cuDNN / flash through
``scaled_dot_product_attention``, flashinfer's fused norm / activation / RoPE
kernels when importable), else the seed in the task dtype. Families follow
the reference's hand-authored directories (kore/tasks/flash_attn_*, gemm_*,
moe_*, fused_*, mla_decode_bf16, paged_attn_decode_bf16, *_backward, and
kore/tasks/vendor_ops.py:183 for genv_*), retargeted to sm_100a: quantised
formats are those B200 executes natively (fp8 e4m3fn, int8, mxfp4 with e8m0
block scales, int4 weights).

Inputs are generated in the task dtype; quantised operands are produced by
quantising random fp32 data with the task's scaling scheme, so oracle and
candidate read the same quantised values and the SNR gate measures the
kernel's arithmetic, not the quantisation error.
"""
from __future__ import annotations

import math
from typing import Callable, Dict, Optional

import torch
import torch.nn.functional as F

from .spec import OpSpec, _gen, _randn

BF = torch.bfloat16
F8 = torch.float8_e4m3fn
F8MAX = 448.0


# ----------------------------------------------------------------------------- helpers
def _ns(src: str) -> dict:
    ns: dict = {}
    exec(src, ns)
    return ns


def _up(x):
    return x.float() if isinstance(x, torch.Tensor) and x.dtype in (torch.bfloat16, torch.float16) else x


def _spec(name, op, entry, src, mk, shapes, family, dtype="bf16", snr=None,
          baseline: Optional[Callable] = None) -> OpSpec:
    fn = _ns(src)[entry]
    ref = lambda *a, fn=fn: _out_f32(fn(*(_up(t) for t in a)))
    return OpSpec(name, op, entry, mk, ref, baseline or fn, src, shapes, family, dtype, snr)


def _out_f32(y):
    return y.float() if isinstance(y, torch.Tensor) and y.is_floating_point() else y


_HDR = "import math\n\nimport torch\nimport torch.nn.functional as F\n\n\n"


def _q8_rows(x, dim=-1):
    """fp8 e4m3fn with one fp32 scale per slice along ``dim`` (amax / 448)."""
    s = x.abs().amax(dim, keepdim=True).clamp_min(1e-8) / F8MAX
    return (x / s).to(F8), s.float()


# ----------------------------------------------------------------------------- attention
_ATTN = _HDR + '''def {entry}(q, k, v{extra}):
    # q [B, H, S, D], k/v [B, KV, Skv, D]; GQA by head groups
    B, H, S, D = q.shape
    KV, Skv = k.shape[1], k.shape[2]
    qf, kf, vf = {load}
    kf = kf.repeat_interleave(H // KV, 1)
    vf = vf.repeat_interleave(H // KV, 1)
    s = (qf @ kf.transpose(-1, -2)) / math.sqrt(D)
    qi = torch.arange(S, device=q.device)[:, None] + (Skv - S)
    ki = torch.arange(Skv, device=q.device)[None, :]
    mask = {mask}
    s = s.masked_fill(~mask, float("-inf"))
{sink}    p = torch.softmax(s, -1)
    return (p @ vf).to({odt})
'''


def _attn_src(entry, causal=True, window=0, sink=False, fp8=False):
    mask = "ki <= qi" if causal else "torch.ones_like(ki <= qi)"
    if window:
        mask = f"(ki <= qi) & (ki > qi - {window})"
    extra = ", sinks" if sink else ""
    extra += ", q_scale, k_scale, v_scale" if fp8 else ""
    load = ("q.float() * q_scale, k.float() * k_scale, v.float() * v_scale" if fp8
            else "q.float(), k.float(), v.float()")
    sink_s = ("    s = torch.cat([s, sinks.float()[None, :, None, None].expand(B, H, S, 1)], -1)\n"
              "    p_all = torch.softmax(s, -1)\n    return (p_all[..., :-1] @ vf).to(q.dtype)\n") if sink else ""
    odt = "torch.bfloat16" if fp8 else "q.dtype"
    return _ATTN.format(entry=entry, extra=extra, load=load, mask=mask, sink=sink_s, odt=odt)


def _mk_attn(fp8=False, sink=False):
    def mk(d, s, dev, dt):
        B, H, S, D = d["B"], d["H"], d["S"], d["D"]
        KV, Skv = d.get("KV", H), d.get("Skv", S)
        q = _randn((B, H, S, D), s, dev, torch.float32)
        k = _randn((B, KV, Skv, D), s + 1, dev, torch.float32)
        v = _randn((B, KV, Skv, D), s + 2, dev, torch.float32)
        if fp8:
            out = []
            for t in (q, k, v):
                sc = t.abs().amax().clamp_min(1e-8) / F8MAX
                out.append(((t / sc).to(F8), sc.reshape(1).float()))
            return out[0][0], out[1][0], out[2][0], out[0][1], out[1][1], out[2][1]
        out = (q.to(dt), k.to(dt), v.to(dt))
        if sink:
            out += (torch.randn(H, generator=_gen(s + 3, dev), device=dev).to(dt),)
        return out
    return mk


def _sdpa_base(causal=True, window=0):
    def base(q, k, v, *rest):
        H, KV = q.shape[1], k.shape[1]
        if window or rest:
            return None
        return F.scaled_dot_product_attention(q, k, v, is_causal=causal and q.shape[2] == k.shape[2],
                                              enable_gqa=H != KV)
    return base


def _attn_task(name, shapes, causal=True, window=0, sink=False, fp8=False, decode=False, snr=None):
    entry = "decode_attention" if decode else "attention"
    src = _attn_src(entry, causal, window, sink, fp8)
    fn = _ns(src)[entry]
    sd = _sdpa_base(causal, window)

    def base(*a, fn=fn, sd=sd):
        r = None if (fp8 or sink or window) else sd(*a)
        return r if r is not None else fn(*a)
    op = "attention_decode" if decode else "attention_prefill"
    return _spec(name, op, entry, src, _mk_attn(fp8, sink), shapes, "attention", "fp8" if fp8 else "bf16",
                 snr or (25.0 if fp8 else 30.0), base)


def _attn_shapes(B, H, KV, S, D, Skv=None, val=()):
    prim = {"B": B, "H": H, "KV": KV, "S": S, "D": D}
    if Skv:
        prim["Skv"] = Skv
    mini = dict(prim, B=1, H=min(H, 4), KV=max(1, min(KV, 4) * min(H, 4) // H) if KV < H else min(H, 4),
                S=min(S, 64), **({"Skv": min(Skv, 128)} if Skv else {}))
    return {"minimal": mini, "primary": prim, "validation": list(val)}


# ----------------------------------------------------------------------------- varlen / backward / paged / mla
_VARLEN = _HDR + '''def {entry}(q, k, v, cu_seqlens):
    # packed q/k/v [T, H|KV, D]; sequences delimited by cu_seqlens (int32 [n + 1])
    T, H, D = q.shape
    KV = k.shape[1]
    out = torch.empty(T, H, D, device=q.device, dtype=torch.float32)
    bounds = cu_seqlens.tolist()
    for a, b in zip(bounds[:-1], bounds[1:]):
        qs = q[a:b].float().transpose(0, 1)
        ks = k[a:b].float().transpose(0, 1).repeat_interleave(H // KV, 0)
        vs = v[a:b].float().transpose(0, 1).repeat_interleave(H // KV, 0)
        s = qs @ ks.transpose(-1, -2) / math.sqrt(D)
        {causal}
        out[a:b] = (torch.softmax(s, -1) @ vs).transpose(0, 1)
    return out.to(q.dtype)
'''


def _mk_varlen(d, s, dev, dt):
    lens = [d["L0"], d["L1"], d["L2"]]
    T = sum(lens)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32, device=dev)
    return (_randn((T, d["H"], d["D"]), s, dev, dt), _randn((T, d["KV"], d["D"]), s + 1, dev, dt),
            _randn((T, d["KV"], d["D"]), s + 2, dev, dt), cu)


_ATTN_BWD = _HDR + '''def attention_backward(q, k, v, do):
    # causal attention backward; returns dq, dk, dv concatenated along the last dim
    qf, kf, vf, dof = q.float(), k.float(), v.float(), do.float()
    D, S = q.shape[-1], q.shape[-2]
    s = qf @ kf.transpose(-1, -2) / math.sqrt(D)
    mask = torch.ones(S, S, dtype=torch.bool, device=q.device).tril()
    p = torch.softmax(s.masked_fill(~mask, float("-inf")), -1)
    dv = p.transpose(-1, -2) @ dof
    dp = dof @ vf.transpose(-1, -2)
    ds = p * (dp - (dp * p).sum(-1, keepdim=True)) / math.sqrt(D)
    dq = ds @ kf
    dk = ds.transpose(-1, -2) @ qf
    return torch.cat([dq, dk, dv], -1).to(q.dtype)
'''

_PAGED = _HDR + '''def paged_attn_decode(q, k_cache, v_cache, block_table, seq_lens):
    # q [B, H, D]; caches [pages, page_size, KV, D]; block_table [B, max_pages] int32
    B, H, D = q.shape
    ps, KV = k_cache.shape[1], k_cache.shape[2]
    out = torch.empty(B, H, D, device=q.device, dtype=torch.float32)
    for b in range(B):
        L = int(seq_lens[b])
        pages = block_table[b, : (L + ps - 1) // ps].long()
        kk = k_cache[pages].reshape(-1, KV, D)[:L].float().repeat_interleave(H // KV, 1)
        vv = v_cache[pages].reshape(-1, KV, D)[:L].float().repeat_interleave(H // KV, 1)
        s = torch.einsum("hd,lhd->hl", q[b].float(), kk) / math.sqrt(D)
        out[b] = torch.einsum("hl,lhd->hd", torch.softmax(s, -1), vv)
    return out.to(q.dtype)
'''


def _mk_paged(d, s, dev, dt):
    B, H, KV, Skv, D, ps = d["B"], d["H"], d["KV"], d["Skv"], d["D"], 16
    npg = (Skv + ps - 1) // ps
    total = B * npg + 3
    perm = torch.randperm(total, generator=_gen(s + 9, "cpu"))[: B * npg].to(torch.int32).reshape(B, npg)
    return (_randn((B, H, D), s, dev, dt), _randn((total, ps, KV, D), s + 1, dev, dt),
            _randn((total, ps, KV, D), s + 2, dev, dt), perm.to(dev),
            torch.full((B,), Skv, dtype=torch.int32, device=dev))


_MLA = _HDR + '''def mla_decode(q_nope, q_rope, kv_latent, k_rope, w_uk, w_uv):
    # absorbed multi-head latent attention (decode):
    # q_nope [B, H, SQ, DNOPE], q_rope [B, H, SQ, DROPE], kv_latent [B, S, DC], k_rope [B, S, DROPE],
    # w_uk [H, DNOPE, DC] (key up-projection), w_uv [H, DC, DV] (value up-projection)
    D = q_nope.shape[-1] + q_rope.shape[-1]
    q_lat = torch.einsum("bhqn,hnc->bhqc", q_nope.float(), w_uk.float())
    s = torch.einsum("bhqc,bsc->bhqs", q_lat, kv_latent.float())
    s = s + torch.einsum("bhqr,bsr->bhqs", q_rope.float(), k_rope.float())
    SQ, S = s.shape[-2], s.shape[-1]
    qi = torch.arange(SQ, device=s.device)[:, None] + (S - SQ)
    s = s.masked_fill(torch.arange(S, device=s.device)[None, :] > qi, float("-inf")) / math.sqrt(D)
    o_lat = torch.einsum("bhqs,bsc->bhqc", torch.softmax(s, -1), kv_latent.float())
    return torch.einsum("bhqc,hcv->bhqv", o_lat, w_uv.float()).to(q_nope.dtype)
'''


def _mk_mla(d, s, dev, dt):
    B, H, S, DC, DN, DR, DV, SQ = (d[k] for k in ("B", "H", "S", "DC", "DNOPE", "DROPE", "DV", "SQ"))
    return (_randn((B, H, SQ, DN), s, dev, dt), _randn((B, H, SQ, DR), s + 1, dev, dt),
            _randn((B, S, DC), s + 2, dev, dt), _randn((B, S, DR), s + 3, dev, dt),
            _randn((H, DN, DC), s + 4, dev, dt, DN ** -0.5), _randn((H, DC, DV), s + 5, dev, dt, DC ** -0.5))


# ----------------------------------------------------------------------------- quantised GEMMs
_GEMM_Q = {
    "gemm_fp8_a8w8": ("a, b, a_scale, b_scale", "(a.float() * a_scale) @ (b.float() * b_scale).t()"),
    "gemm_fp8_a8w8_pertensor": ("a, b, a_scale, b_scale", "(a.float() * a_scale) @ (b.float() * b_scale).t()"),
    "gemm_fp8_a8w8_pertoken": ("a, b, a_scale, b_scale",
                               "(a.float() @ b.float().t()) * a_scale * b_scale.t()"),
    "gemm_int8_a8w8": ("a, b, a_scale, b_scale", "(a.float() @ b.float().t()) * a_scale * b_scale.t()"),
    "gemm_fp8_a8w8_blockscale": ("a, b, a_scale, b_scale",
                                 "(a.float() * a_scale.repeat_interleave(128, 1)) @ "
                                 "(b.float() * b_scale.repeat_interleave(128, 0).repeat_interleave(128, 1)).t()"),
    "gemm_fp8_requant_epilogue": ("a, b, a_scale, b_scale, out_scale",
                                  "((a.float() * a_scale) @ (b.float() * b_scale).t() / out_scale)"
                                  ".clamp(-448.0, 448.0)"),
    "gemm_w4a16": ("a, b_packed, b_scale", "a.float() @ (_unpack_int4(b_packed) * b_scale).t()"),
    "gemm_w4a16_g128": ("a, b_packed, b_scale",
                        "a.float() @ (_unpack_int4(b_packed) * b_scale.repeat_interleave(128, 1)).t()"),
    "gemm_w4a8_fp8": ("a, b_packed, a_scale, b_scale",
                      "(a.float() * a_scale) @ (_unpack_int4(b_packed) * b_scale).t()"),
    "gemm_mxfp4": ("a, b_packed, b_scale_e8m0",
                   "a.float() @ (_unpack_fp4(b_packed) * _e8m0(b_scale_e8m0).repeat_interleave(32, 1)).t()"),
    "gemm_mxfp4_a4w4": ("a_packed, a_scale_e8m0, b_packed, b_scale_e8m0",
                        "(_unpack_fp4(a_packed) * _e8m0(a_scale_e8m0).repeat_interleave(32, 1)) @ "
                        "(_unpack_fp4(b_packed) * _e8m0(b_scale_e8m0).repeat_interleave(32, 1)).t()"),
}
_Q_HELPERS = '''_FP4 = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0])


def _unpack_int4(p):
    # two signed 4-bit values per byte, low nibble first
    lo = (p & 0xF).to(torch.int16)
    hi = ((p >> 4) & 0xF).to(torch.int16)
    v = torch.stack([lo, hi], -1).reshape(p.shape[0], -1)
    return torch.where(v >= 8, v - 16, v).float()


def _unpack_fp4(p):
    # two e2m1 codes per byte, low nibble first
    idx = torch.stack([(p & 0xF).long(), ((p >> 4) & 0xF).long()], -1).reshape(p.shape[0], -1)
    return _FP4.to(p.device)[idx]


def _e8m0(s):
    return torch.exp2(s.float() - 127.0)


'''


def _pack_nibbles(v):
    v = v.to(torch.int16) & 0xF
    return (v[:, 0::2] | (v[:, 1::2] << 4)).to(torch.uint8)


def _fp4_codes(x):
    grid = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], device=x.device)
    mag = (x.abs()[..., None] - grid).abs().argmin(-1)
    return torch.where(x < 0, mag + 8, mag)


def _mxfp4(x):
    """[R, K] fp32 -> (packed e2m1 codes [R, K/2] uint8, e8m0 scale per 32 [R, K/32] uint8)."""
    R, K = x.shape
    blocks = x.reshape(R, K // 32, 32)
    e = torch.floor(torch.log2(blocks.abs().amax(-1).clamp_min(1e-30) / 6.0)).clamp(-127, 127)
    codes = _fp4_codes((blocks / torch.exp2(e)[..., None]).reshape(R, K))
    return _pack_nibbles(codes), (e + 127).to(torch.uint8)


def _mk_qgemm(kind):
    def mk(d, s, dev, dt):
        M, N, K = d["M"], d["N"], d["K"]
        a = _randn((M, K), s, dev, torch.float32)
        b = _randn((N, K), s + 1, dev, torch.float32, K ** -0.5)
        if kind in ("gemm_fp8_a8w8", "gemm_fp8_a8w8_pertensor", "gemm_fp8_requant_epilogue"):
            sa, sb = a.abs().amax() / F8MAX, b.abs().amax() / F8MAX
            out = ((a / sa).to(F8), (b / sb).to(F8), sa.reshape(1, 1), sb.reshape(1, 1))
            if kind == "gemm_fp8_requant_epilogue":
                out += (torch.tensor([[0.05]], device=dev),)
            return out
        if kind == "gemm_fp8_a8w8_pertoken":
            qa, sa = _q8_rows(a)
            qb, sb = _q8_rows(b)
            return qa, qb, sa, sb
        if kind == "gemm_int8_a8w8":
            sa = a.abs().amax(-1, keepdim=True) / 127
            sb = b.abs().amax(-1, keepdim=True) / 127
            return (a / sa).round().to(torch.int8), (b / sb).round().to(torch.int8), sa, sb
        if kind == "gemm_fp8_a8w8_blockscale":
            sa = a.reshape(M, K // 128, 128).abs().amax(-1) / F8MAX
            sb = b.reshape(N // 128, 128, K // 128, 128).abs().amax((1, 3)) / F8MAX
            qa = (a / sa.repeat_interleave(128, 1)).to(F8)
            qb = (b / sb.repeat_interleave(128, 0).repeat_interleave(128, 1)).to(F8)
            return qa, qb, sa, sb
        if kind in ("gemm_w4a16", "gemm_w4a16_g128", "gemm_w4a8_fp8"):
            if kind == "gemm_w4a16_g128":
                sb = b.reshape(N, K // 128, 128).abs().amax(-1) / 7
                q = (b / sb.repeat_interleave(128, 1)).round().clamp(-8, 7)
            else:
                sb = b.abs().amax(-1, keepdim=True) / 7
                q = (b / sb).round().clamp(-8, 7)
            packed = _pack_nibbles(q)
            if kind == "gemm_w4a8_fp8":
                saa = a.abs().amax() / F8MAX
                return (a / saa).to(F8), packed, saa.reshape(1, 1), sb
            return a.to(dt), packed, sb
        if kind == "gemm_mxfp4":
            pb, eb = _mxfp4(b)
            return a.to(dt), pb, eb
        if kind == "gemm_mxfp4_a4w4":
            pa, ea = _mxfp4(a)
            pb, eb = _mxfp4(b)
            return pa, ea, pb, eb
        raise KeyError(kind)
    return mk


def _qgemm_task(kind):
    args, expr = _GEMM_Q[kind]
    src = _HDR + _Q_HELPERS + f"def {kind}({args}):\n    return ({expr}).to(torch.bfloat16)\n"
    if kind == "gemm_fp8_requant_epilogue":
        src = _HDR + _Q_HELPERS + f"def {kind}({args}):\n    return ({expr}).to(torch.float8_e4m3fn)\n"
    shapes = {"minimal": {"M": 128, "N": 256, "K": 256}, "primary": {"M": 4096, "N": 4096, "K": 4096},
              "validation": [{"M": 1, "N": 4096, "K": 4096}, {"M": 2048, "N": 14336, "K": 4096},
                             {"M": 8, "N": 7168, "K": 2048}]}
    dt = "fp8" if "fp8" in kind else ("int8" if "int8" in kind else ("fp4" if "mxfp4" in kind else "int4"))
    return _spec(kind, kind, kind, src, _mk_qgemm(kind), shapes, "gemm_quant", dt, 25.0)


_GEMM_BWD = _HDR + '''def gemm_backward(a, b, dc):
    # C = A B^T; returns dA = dC B and dB = dC^T A, flattened and concatenated
    da = dc.float() @ b.float()
    db = dc.float().t() @ a.float()
    return torch.cat([da.reshape(-1), db.reshape(-1)]).to(a.dtype)
'''


# ----------------------------------------------------------------------------- MoE
_MOE = _HDR + '''def {entry}(x, router_logits, w_gate_up, w_down{extra}):
    # x [M, D]; router_logits [M, E]; w_gate_up [E, 2I, D]; w_down [E, D, I]
    {route}
    M, D = x.shape
    out = torch.zeros(M, D, device=x.device, dtype=torch.float32)
    xf = x.float()
    for e in range(w_gate_up.shape[0]):
        rows, slot = (idx == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        gu = xf[rows] @ w_gate_up[e].float().t()
        g, u = gu.chunk(2, -1)
        h = {act} * u
        out.index_add_(0, rows, (h @ w_down[e].float().t()) * wts[rows, slot, None])
    return out.to(x.dtype)
'''
_ROUTE_SOFTMAX = ("p = torch.softmax(router_logits.float(), -1)\n    wts, idx = p.topk(TOPK, -1)\n"
                  "    wts = wts / wts.sum(-1, keepdim=True)")


def _mk_moe(d, s, dev, dt):
    M, E, D, I = d["M"], d["E"], d["D"], d["I"]
    return (_randn((M, D), s, dev, dt), _randn((M, E), s + 1, dev, torch.float32),
            _randn((E, 2 * I, D), s + 2, dev, dt, D ** -0.5), _randn((E, D, I), s + 3, dev, dt, I ** -0.5))


def _moe_src(entry, act, topk):
    return _MOE.format(entry=entry, extra="", route=_ROUTE_SOFTMAX.replace("TOPK", str(topk)),
                       act={"silu": "F.silu(g)", "gelu": "F.gelu(g, approximate='tanh')"}[act])


_MOE_SMALL = {
    "moe_topk_softmax_norenorm": ("logits", "p = torch.softmax(logits.float(), -1)\n    w, i = p.topk(8, -1)\n"
                                  "    return torch.cat([w, i.float()], -1)"),
    "moe_biased_grouped_topk": ("logits, bias",
                                "# DeepSeek-V3: sigmoid scores, bias for selection only, 8 groups, top-4 groups\n"
                                "    sc = torch.sigmoid(logits.float())\n    sel = sc + bias.float()\n"
                                "    M, E = sel.shape\n    g = sel.reshape(M, 8, E // 8).topk(2, -1).values.sum(-1)\n"
                                "    keep = torch.zeros_like(g).scatter(1, g.topk(4, -1).indices, 1.0)\n"
                                "    sel = sel.masked_fill(keep.repeat_interleave(E // 8, 1) == 0, float('-inf'))\n"
                                "    i = sel.topk(8, -1).indices\n    w = sc.gather(1, i)\n"
                                "    w = w / w.sum(-1, keepdim=True) * 2.5\n    return torch.cat([w, i.float()], -1)"),
    "moe_permute": ("x, topk_ids", "# rows grouped by expert (stable by token), one row per (token, slot)\n"
                    "    M, k = topk_ids.shape\n    flat = topk_ids.reshape(-1)\n"
                    "    order = torch.argsort(flat * (M * k) + torch.arange(M * k, device=x.device))\n"
                    "    return x.float()[order // k]"),
    "moe_sum_combine": ("expert_out, topk_weights", "# expert_out [M, k, D] -> weighted sum over k\n"
                        "    return (expert_out.float() * topk_weights.float()[..., None]).sum(1)"),
    "moe_batched_gemm": ("a, b", "# a [E, M, K], b [E, N, K]\n    return torch.bmm(a.float(), b.float().transpose(1, 2))"),
    "moe_grouped_gemm": ("a, b, offsets", "# rows of a grouped by expert: [offsets[e], offsets[e+1]) use b[e]\n"
                         "    out = torch.empty(a.shape[0], b.shape[1], device=a.device)\n"
                         "    o = offsets.tolist()\n    for e in range(b.shape[0]):\n"
                         "        out[o[e]:o[e + 1]] = a[o[e]:o[e + 1]].float() @ b[e].float().t()\n    return out"),
    "moe_grouped_gemm_fp8": ("a, b, a_scale, b_scale, offsets",
                             "out = torch.empty(a.shape[0], b.shape[1], device=a.device)\n    o = offsets.tolist()\n"
                             "    for e in range(b.shape[0]):\n"
                             "        out[o[e]:o[e + 1]] = (a[o[e]:o[e + 1]].float() * a_scale[o[e]:o[e + 1]]) @ "
                             "(b[e].float() * b_scale[e]).t()\n    return out"),
}


def _mk_moe_small(name):
    def mk(d, s, dev, dt):
        M, E = d.get("M", 256), d.get("E", 64)
        if name == "moe_topk_softmax_norenorm":
            return (_randn((M, E), s, dev, dt),)
        if name == "moe_biased_grouped_topk":
            return _randn((M, E), s, dev, dt), _randn((E,), s + 1, dev, dt, 0.1)
        if name == "moe_permute":
            ids = torch.randint(0, E, (M, 8), generator=_gen(s, dev), device=dev)
            return _randn((M, d["D"]), s, dev, dt), ids
        if name == "moe_sum_combine":
            w = torch.softmax(_randn((M, 8), s + 1, dev, torch.float32), -1).to(dt)
            return _randn((M, 8, d["D"]), s, dev, dt), w
        if name == "moe_batched_gemm":
            return (_randn((E, d["M"], d["K"]), s, dev, dt), _randn((E, d["N"], d["K"]), s + 1, dev, dt,
                                                                      d["K"] ** -0.5))
        counts = torch.randint(0, 2 * d["M"] // E + 1, (E,), generator=_gen(s, "cpu"))
        offs = torch.cat([torch.zeros(1, dtype=torch.long), counts.cumsum(0)]).to(torch.int32)
        T = int(offs[-1])
        a = _randn((T, d["K"]), s + 1, dev, torch.float32)
        b = _randn((E, d["N"], d["K"]), s + 2, dev, torch.float32, d["K"] ** -0.5)
        if name == "moe_grouped_gemm_fp8":
            qa, sa = _q8_rows(a)
            sb = b.abs().amax((1, 2)).reshape(E, 1, 1) / F8MAX
            return qa, (b / sb).to(F8), sa, sb.reshape(E, 1), offs.to(dev)
        return a.to(dt), b.to(dt), offs.to(dev)
    return mk


# ----------------------------------------------------------------------------- fused / backward
_FUSED = {
    "fused_add_rmsnorm": ("x, residual, w", "h = x.float() + residual.float()\n"
                          "    y = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()\n"
                          "    return torch.cat([y, h], -1).to(x.dtype)"),
    "fused_rmsnorm_quant_fp8": ("x, w", "y = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)"
                                " * w.float()\n    s = y.abs().amax(-1, keepdim=True).clamp_min(1e-8) / 448.0\n"
                                "    return torch.cat([(y / s).to(torch.float8_e4m3fn).float(), s], -1)"),
    "fused_silu_mul_quant_fp8": ("a, b", "y = F.silu(a.float()) * b.float()\n"
                                 "    s = y.abs().amax(-1, keepdim=True).clamp_min(1e-8) / 448.0\n"
                                 "    return torch.cat([(y / s).to(torch.float8_e4m3fn).float(), s], -1)"),
    "rmsnorm_backward": ("x, w, dy", "xf, wf, g = x.float(), w.float(), dy.float()\n"
                         "    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)\n"
                         "    gw = g * wf\n    dx = r * (gw - xf * r * r * (gw * xf).mean(-1, keepdim=True))\n"
                         "    dw = (g * xf * r).sum(0, keepdim=True)\n    return torch.cat([dx, dw], 0).to(x.dtype)"),
    "layernorm_backward": ("x, w, dy", "xf, wf, g = x.float(), w.float(), dy.float()\n"
                           "    mu = xf.mean(-1, keepdim=True)\n"
                           "    r = torch.rsqrt(((xf - mu) ** 2).mean(-1, keepdim=True) + 1e-5)\n"
                           "    xh = (xf - mu) * r\n    gw = g * wf\n"
                           "    dx = r * (gw - gw.mean(-1, keepdim=True) - xh * (gw * xh).mean(-1, keepdim=True))\n"
                           "    dw = (g * xh).sum(0, keepdim=True)\n    return torch.cat([dx, dw], 0).to(x.dtype)"),
    "softmax_backward": ("y, dy", "# y = softmax(x); returns dx\n"
                         "    yf, g = y.float(), dy.float()\n    return (yf * (g - (g * yf).sum(-1, keepdim=True))).to(y.dtype)"),
}


def _mk_fused(name):
    def mk(d, s, dev, dt):
        M, N = d["M"], d["N"]
        x = _randn((M, N), s, dev, dt)
        w = (1 + 0.1 * _randn((N,), s + 1, dev, torch.float32)).to(dt)
        if name == "fused_add_rmsnorm":
            return x, _randn((M, N), s + 2, dev, dt), w
        if name == "fused_rmsnorm_quant_fp8":
            return x, w
        if name == "fused_silu_mul_quant_fp8":
            return x, _randn((M, N), s + 2, dev, dt)
        if name == "softmax_backward":
            return torch.softmax(x.float(), -1).to(dt), _randn((M, N), s + 2, dev, dt)
        return x, w, _randn((M, N), s + 2, dev, dt)
    return mk


# ----------------------------------------------------------------------------- vendor ops (genv_*)
def _fi(name):
    try:
        import flashinfer
        return getattr(flashinfer, name, None)
    except Exception:  # noqa: BLE001 - flashinfer is an optional vendor baseline
        return None


_GENV = {
    "rmsnorm": ("x, w", "return (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)"
                " * w.float()).to(x.dtype)", "rmsnorm"),
    "fused_add_rmsnorm": ("x, residual, w", "h = x.float() + residual.float()\n    return torch.cat([(h * "
                          "torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()), h], -1).to(x.dtype)",
                          None),
    "layernorm": ("x, w, b", "return F.layer_norm(x.float(), (x.shape[-1],), w.float(), b.float(), 1e-5)"
                  ".to(x.dtype)", None),
    "silu_mul": ("x", "g, u = x.float().chunk(2, -1)\n    return (F.silu(g) * u).to(x.dtype)", "silu_and_mul"),
    "gelu_mul": ("x", "g, u = x.float().chunk(2, -1)\n    return (F.gelu(g, approximate='tanh') * u).to(x.dtype)",
                 "gelu_tanh_and_mul"),
    "softmax": ("x", "return torch.softmax(x.float(), -1).to(x.dtype)", None),
    "topk_softmax": ("logits", "p = torch.softmax(logits.float(), -1)\n    w, i = p.topk(8, -1)\n"
                     "    return torch.cat([w / w.sum(-1, keepdim=True), i.float()], -1)", None),
    "embedding_gather": ("table, ids", "return table[ids.long()]", None),
    "rope": ("x, cos, sin", "# NeoX rotation (halves); x [T, H, D], cos/sin [T, D/2]\n"
             "    d = x.shape[-1] // 2\n    x1, x2 = x.float()[..., :d], x.float()[..., d:]\n"
             "    c, s = cos.float()[:, None], sin.float()[:, None]\n"
             "    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).to(x.dtype)", None),
    "rope_gptj": ("x, cos, sin", "# GPT-J rotation (interleaved pairs)\n"
                  "    x1, x2 = x.float()[..., 0::2], x.float()[..., 1::2]\n"
                  "    c, s = cos.float()[:, None], sin.float()[:, None]\n"
                  "    return torch.stack([x1 * c - x2 * s, x2 * c + x1 * s], -1).flatten(-2).to(x.dtype)", None),
    "rope_partial": ("x, cos, sin", "# rotate the first 64 dims (NeoX halves), pass the rest through\n"
                     "    r, p = x.float()[..., :64], x.float()[..., 64:]\n    x1, x2 = r[..., :32], r[..., 32:]\n"
                     "    c, s = cos.float()[:, None], sin.float()[:, None]\n"
                     "    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s, p], -1).to(x.dtype)", None),
    "batched_gemm": ("a, b", "return torch.bmm(a.float(), b.float().transpose(1, 2)).to(a.dtype)", None),
}


def _mk_genv(name):
    def mk(d, s, dev, dt):
        M, N = d.get("M", 4096), d.get("N", 4096)
        if name in ("rmsnorm",):
            return _randn((M, N), s, dev, dt), (1 + 0.1 * _randn((N,), s + 1, dev, torch.float32)).to(dt)
        if name == "fused_add_rmsnorm":
            return (_randn((M, N), s, dev, dt), _randn((M, N), s + 2, dev, dt),
                    (1 + 0.1 * _randn((N,), s + 1, dev, torch.float32)).to(dt))
        if name == "layernorm":
            return (_randn((M, N), s, dev, dt), (1 + 0.1 * _randn((N,), s + 1, dev, torch.float32)).to(dt),
                    _randn((N,), s + 3, dev, dt, 0.1))
        if name in ("silu_mul", "gelu_mul"):
            return (_randn((M, 2 * N), s, dev, dt),)
        if name == "softmax":
            return (_randn((M, N), s, dev, dt),)
        if name == "topk_softmax":
            return (_randn((M, d.get("E", 128)), s, dev, dt),)
        if name == "embedding_gather":
            return (_randn((d["V"], N), s, dev, dt), torch.randint(0, d["V"], (M,), generator=_gen(s, dev),
                                                                    device=dev))
        if name.startswith("rope"):
            T, H, D = d["T"], d["H"], d["D"]
            half = 32 if name == "rope_partial" else D // 2
            ang = torch.arange(T, device=dev, dtype=torch.float32)[:, None] * \
                torch.exp2(-torch.arange(half, device=dev, dtype=torch.float32) / half * 13.3)[None]
            return _randn((T, H, D), s, dev, dt), ang.cos().to(dt), ang.sin().to(dt)
        if name == "batched_gemm":
            return (_randn((d["B"], d["M"], d["K"]), s, dev, dt),
                    _randn((d["B"], d["N"], d["K"]), s + 1, dev, dt, d["K"] ** -0.5))
        raise KeyError(name)
    return mk


_GENV_SHAPES = {
    "rope": {"minimal": {"T": 16, "H": 4, "D": 128}, "primary": {"T": 8192, "H": 32, "D": 128},
             "validation": [{"T": 1, "H": 8, "D": 128}, {"T": 4097, "H": 40, "D": 128}]},
    "embedding_gather": {"minimal": {"M": 16, "N": 256, "V": 1000},
                         "primary": {"M": 8192, "N": 5120, "V": 151936},
                         "validation": [{"M": 1, "N": 4096, "V": 32000}]},
    "batched_gemm": {"minimal": {"B": 2, "M": 64, "N": 64, "K": 64},
                     "primary": {"B": 32, "M": 1024, "N": 1024, "K": 128},
                     "validation": [{"B": 8, "M": 4096, "N": 128, "K": 4096}]},
    "topk_softmax": {"minimal": {"M": 16, "E": 64}, "primary": {"M": 8192, "E": 128},
                     "validation": [{"M": 1, "E": 256}]},
}
_ROWS = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 8192, "N": 5120},
         "validation": [{"M": 1, "N": 4096}, {"M": 333, "N": 8192}]}


def _genv_task(name, dt):
    args, body, fi_name = _GENV[name]
    src = _HDR + f"def {name}({args}):\n    {body}\n"
    base = None
    if fi_name is not None:
        fn = _ns(src)[name]

        def base(*a, fn=fn, fi_name=fi_name):
            f = _fi(fi_name) if a[0].is_cuda else None
            if f is None:
                return fn(*a)
            return f(*a, 1e-6) if fi_name == "rmsnorm" else f(*a)
    key = "rope" if name.startswith("rope") else name
    shapes = _GENV_SHAPES.get(key, _ROWS)
    op = {"silu_mul": "silu_mul", "gelu_mul": "gelu_mul", "rmsnorm": "rmsnorm", "fused_add_rmsnorm":
          "fused_add_rmsnorm", "layernorm": "layernorm", "softmax": "softmax", "topk_softmax": "topk_router",
          "batched_gemm": "batched_gemm"}.get(name, "rope" if key == "rope" else name)
    return _spec(f"genv_{name}_{dt}", op, name, src, _mk_genv(name), shapes, "vendor", dt, 30.0, base)


# ----------------------------------------------------------------------------- registry
def build() -> Dict[str, OpSpec]:
    out: Dict[str, OpSpec] = {}

    def add(s: OpSpec):
        out[s.name] = s

    # attention family (17 with the two core tasks in ops_library)
    add(_attn_task("flash_attn_mha_prefill_bf16", _attn_shapes(1, 32, 32, 2048, 128)))
    add(_attn_task("flash_attn_mqa_prefill_bf16", _attn_shapes(1, 32, 1, 2048, 128)))
    add(_attn_task("flash_attn_noncausal_prefill_bf16", _attn_shapes(1, 32, 8, 2048, 128), causal=False))
    add(_attn_task("flash_attn_headdim_prefill_bf16", _attn_shapes(1, 16, 4, 2048, 256,
                                                                    val=[{"B": 1, "H": 32, "KV": 8, "S": 2048, "D": 64}])))
    add(_attn_task("flash_attn_sink_prefill_bf16", _attn_shapes(1, 32, 8, 2048, 128), sink=True))
    add(_attn_task("flash_attn_sliding_bf16", _attn_shapes(1, 32, 8, 4096, 128), window=1024))
    add(_attn_task("flash_attn_chunked_prefill_bf16", _attn_shapes(1, 32, 8, 512, 128, Skv=4096)))
    add(_attn_task("flash_attn_fp8_bf16", _attn_shapes(1, 32, 8, 2048, 128), fp8=True))
    add(_attn_task("flash_attn_noncausal_fp8", _attn_shapes(1, 32, 8, 2048, 128), causal=False, fp8=True))
    add(_attn_task("flash_attn_mqa_decode_bf16", _attn_shapes(8, 32, 1, 1, 128, Skv=4096), decode=True))
    add(_attn_task("flash_attn_sliding_decode_bf16", _attn_shapes(8, 32, 8, 1, 128, Skv=8192), window=4096,
                   decode=True))
    add(_attn_task("flash_attn_decode_fp8", _attn_shapes(8, 32, 8, 1, 128, Skv=4096), fp8=True, decode=True))
    for nm, causal in (("flash_attn_varlen_bf16", True), ("flash_attn_varlen_noncausal_bf16", False)):
        src = _VARLEN.format(entry="varlen_attention", causal=(
            "s = s.masked_fill(torch.ones_like(s, dtype=torch.bool).triu(1), float('-inf'))" if causal else "pass"))
        add(_spec(nm, "attention_prefill", "varlen_attention", src, _mk_varlen,
                  {"minimal": {"L0": 17, "L1": 64, "L2": 5, "H": 4, "KV": 2, "D": 128},
                   "primary": {"L0": 2048, "L1": 1000, "L2": 3100, "H": 32, "KV": 8, "D": 128, "B": 3, "S": 2048},
                   "validation": [{"L0": 1, "L1": 4096, "L2": 1, "H": 32, "KV": 8, "D": 128}]}, "attention"))
    add(_spec("flash_attn_backward_bf16", "attention_prefill", "attention_backward", _ATTN_BWD,
              lambda d, s, dev, dt: tuple(_randn((d["B"], d["H"], d["S"], d["D"]), s + i, dev, dt) for i in range(4)),
              {"minimal": {"B": 1, "H": 2, "S": 64, "D": 128}, "primary": {"B": 1, "H": 32, "S": 2048, "D": 128},
               "validation": [{"B": 2, "H": 8, "S": 1000, "D": 128}]}, "attention"))
    add(_spec("paged_attn_decode_bf16", "attention_decode", "paged_attn_decode", _PAGED, _mk_paged,
              {"minimal": {"B": 1, "H": 8, "KV": 2, "Skv": 256, "D": 128},
               "primary": {"B": 8, "H": 32, "KV": 8, "Skv": 4096, "D": 128},
               "validation": [{"B": 1, "H": 32, "KV": 8, "Skv": 8192, "D": 128},
                              {"B": 4, "H": 32, "KV": 8, "Skv": 1000, "D": 128}]}, "attention", snr=25.0))
    add(_spec("mla_decode_bf16", "mla_decode", "mla_decode", _MLA, _mk_mla,
              {"minimal": {"B": 1, "H": 4, "S": 256, "DC": 512, "DNOPE": 128, "DROPE": 64, "DV": 128, "SQ": 1},
               "primary": {"B": 1, "H": 16, "S": 2048, "DC": 512, "DNOPE": 128, "DROPE": 64, "DV": 128, "SQ": 1},
               "validation": [{"B": 2, "H": 8, "S": 2048, "DC": 512, "DNOPE": 128, "DROPE": 64, "DV": 128,
                               "SQ": 16}]}, "mla", snr=25.0))
    # GEMM family
    for kind in _GEMM_Q:
        add(_qgemm_task(kind))
    add(_spec("gemm_backward_bf16", "gemm", "gemm_backward", _GEMM_BWD,
              lambda d, s, dev, dt: (_randn((d["M"], d["K"]), s, dev, dt), _randn((d["N"], d["K"]), s + 1, dev, dt),
                                     _randn((d["M"], d["N"]), s + 2, dev, dt)),
              {"minimal": {"M": 64, "N": 128, "K": 64}, "primary": {"M": 4096, "N": 4096, "K": 4096},
               "validation": [{"M": 8192, "N": 5120, "K": 1024}]}, "gemm"))
    # MoE family
    moe_shapes = {"minimal": {"M": 32, "E": 8, "D": 128, "I": 64}, "primary": {"M": 256, "E": 32, "D": 1024, "I": 768},
                  "validation": [{"M": 4096, "E": 128, "D": 2048, "I": 768}]}
    add(_spec("fused_moe_silu_bf16", "moe", "fused_moe", _moe_src("fused_moe", "silu", 8).replace("TOPK", "8"),
              _mk_moe, moe_shapes, "moe"))
    add(_spec("moe_gelu_bf16", "moe", "moe_gelu", _moe_src("moe_gelu", "gelu", 8), _mk_moe, moe_shapes, "moe"))
    small_shapes = {"minimal": {"M": 64, "E": 64, "D": 128, "N": 64, "K": 64},
                    "primary": {"M": 8192, "E": 128, "D": 2048, "N": 1536, "K": 2048},
                    "validation": [{"M": 1, "E": 256, "D": 7168, "N": 512, "K": 7168}]}
    for nm, (args, body) in _MOE_SMALL.items():
        add(_spec(f"{nm}_bf16" if not nm.endswith("fp8") else nm, "moe_" + nm.split("moe_")[-1], nm,
                  _HDR + f"def {nm}({args}):\n    {body}\n", _mk_moe_small(nm), small_shapes, "moe",
                  "fp8" if nm.endswith("fp8") else "bf16", 25.0))
    # fused + backward
    fshapes = {"minimal": {"M": 16, "N": 1024}, "primary": {"M": 8192, "N": 5120},
               "validation": [{"M": 1, "N": 8192}, {"M": 333, "N": 4096}]}
    for nm, (args, body) in _FUSED.items():
        tid = nm + ("_bf16" if not nm.endswith("fp8") else "")
        add(_spec(tid, nm, nm, _HDR + f"def {nm}({args}):\n    {body}\n", _mk_fused(nm), fshapes,
                  "fused" if nm.startswith("fused") else "norm", "fp8" if nm.endswith("fp8") else "bf16",
                  25.0 if nm.endswith("fp8") else 30.0))
    # vendor ops
    for dt in ("bf16", "fp16"):
        for nm in ("rmsnorm", "fused_add_rmsnorm", "layernorm", "silu_mul", "gelu_mul", "softmax", "topk_softmax",
                   "embedding_gather", "rope", "rope_gptj", "rope_partial"):
            add(_genv_task(nm, dt))
    add(_genv_task("batched_gemm", "bf16"))
    for alias, kind in (("genv_gemm_a8w8_fp8", "gemm_fp8_a8w8_pertoken"), ("genv_gemm_a8w8_int8", "gemm_int8_a8w8"),
                        ("genv_gemm_a8w8_blockscale_fp8", "gemm_fp8_a8w8_blockscale")):
        q = _qgemm_task(kind)
        q.name, q.family = alias, "vendor"
        add(q)
    return out
