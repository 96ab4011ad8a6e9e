"""Expert parallelism: MoE tokens are dispatched to the rank that owns their
experts and the expert outputs are combined back.

Each rank owns experts [lo, hi) (``Qwen3Weights(ep=(rank, world))``) and its
own tokens. Forward of one MoE layer:

  local route -> pairs sorted by global expert (so rows for each destination
  rank are contiguous) -> exchange per-expert counts -> all-to-all of the
  token rows -> expert-major permutation of the received rows -> grouped
  tcgen05 GEMMs (SwiGLU experts) -> inverse permutation -> all-to-all back
  -> weighted combine (+ residual) at the source.

The backward mirrors it (combine bwd -> all-to-all -> expert backward with
local weight gradients -> all-to-all -> un-permute sum). Data planes:
``comm="nccl"`` uses ``all_to_all_single``; the counts are needed on the
host anyway to size the grouped GEMM. Expert weights and their gradients
never leave their rank; only the replicated parts go through ZeRO.
"""
from __future__ import annotations

from typing import List, Tuple

import torch
import torch.distributed as dist

from .. import ops
from ..ops import moe


class ExpertParallel:
    def __init__(self, ctx, cfg, lo: int, hi: int):
        self.ctx = ctx
        self.cfg = cfg
        self.lo, self.hi = lo, hi
        self.W = ctx.world
        self.E = cfg.num_experts
        self.El = hi - lo

    # ------------------------------------------------------------ plumbing
    def _a2a(self, x: torch.Tensor, send: List[int], recv: List[int]) -> torch.Tensor:
        out = torch.empty((sum(recv),) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        if self.ctx.backend == "nccl":
            dist.all_to_all_single(out, x.contiguous(), recv, send, group=self.ctx.group)
        else:  # gloo: no all_to_all_single on CPU for every dtype -> gather-based exchange
            chunks = list(x.split(send))
            gathered = [None] * self.W
            dist.all_gather_object(gathered, [c.cpu() for c in chunks], group=self.ctx.group)
            parts = [gathered[s][self.ctx.rank].to(x.device) for s in range(self.W)]
            out = torch.cat(parts) if parts else out
        return out

    def _plan(self, idx: torch.Tensor):
        """Send order (pairs sorted by global expert), per-dest row counts, and the
        receive-side counts matrix [src, local expert]."""
        T, k = idx.shape
        flat = idx.reshape(-1).long()
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=self.E)               # [E] on this rank
        cm = torch.empty(self.W * self.El, dtype=counts.dtype, device=counts.device)
        if self.ctx.backend == "nccl":
            dist.all_to_all_single(cm, counts.contiguous(), group=self.ctx.group)
        else:
            g = [None] * self.W
            dist.all_gather_object(g, counts.cpu(), group=self.ctx.group)
            cm = torch.cat([g[s][self.lo:self.hi] for s in range(self.W)]).to(counts.device)
        cnt = counts.view(self.W, self.El).sum(1).tolist()             # rows to each dest
        recv_mat = cm.view(self.W, self.El).tolist()                   # [src][local expert]
        return order, cnt, recv_mat

    @staticmethod
    def _expert_major(recv_mat) -> Tuple[torch.Tensor, List[int]]:
        """Permutation from src-major receive order to expert-major order."""
        W = len(recv_mat)
        El = len(recv_mat[0]) if W else 0
        src_off, o = [], 0
        base = [[0] * El for _ in range(W)]
        for s in range(W):
            for e in range(El):
                base[s][e] = o
                o += recv_mat[s][e]
        perm, offs = [], [0]
        for e in range(El):
            for s in range(W):
                perm.extend(range(base[s][e], base[s][e] + recv_mat[s][e]))
            offs.append(len(perm))
        return torch.tensor(perm, dtype=torch.long), offs

    # ------------------------------------------------------------ forward
    def forward(self, eng, W, hn2, x2, probs, idx, wts):
        T, k = idx.shape
        order, send, recv_mat = self._plan(idx)
        recv = [sum(r) for r in recv_mat]
        rows = moe.gather_rows(hn2, order // k)                         # send buffer
        xr = self._a2a(rows, send, recv)
        perm, offs = self._expert_major(recv_mat)
        perm = perm.to(hn2.device)
        xp = moe.gather_rows(xr, perm)
        gu = moe.grouped_mm(xp, W["experts_gate_up"], offs)
        a = ops.swiglu_fwd(gu)
        yp = moe.grouped_mm(a, W["experts_down"], offs)
        yr = torch.empty_like(yp)
        yr[perm] = yp                                                   # back to src-major
        ys = self._a2a(yr, recv, send)                                  # rows in send order
        pos = torch.empty(T * k, dtype=torch.int32, device=hn2.device)
        pos[order] = torch.arange(T * k, dtype=torch.int32, device=hn2.device)
        pos = pos.view(T, k)
        x3 = moe.combine(ys, pos, wts, resid=x2)
        ctx = dict(probs=probs, idx=idx, wts=wts, pos=pos, order=order, send=send, recv=recv, perm=perm,
                   offs=offs, xp=xp, gu=gu, a=a, ys=ys)
        return x3, ctx

    # ------------------------------------------------------------ backward
    def backward(self, eng, W, G, ctx, dx3):
        dys, dw = moe.combine_bwd(dx3, ctx["ys"], ctx["pos"], ctx["wts"])
        dyr = self._a2a(dys, ctx["send"], ctx["recv"])
        dyp = moe.gather_rows(dyr, ctx["perm"])
        offs = ctx["offs"]
        da = moe.grouped_mm(dyp, W["experts_down"], offs, w_t=False)
        eng._expert_wgrad(G["experts_down"], dyp, ctx["a"], offs)
        dgu = ops.swiglu_bwd(da, ctx["gu"], ctx["gu"])
        dxp = moe.grouped_mm(dgu, W["experts_gate_up"], offs, w_t=False)
        eng._expert_wgrad(G["experts_gate_up"], dgu, ctx["xp"], offs)
        dxr = torch.empty_like(dxp)
        dxr[ctx["perm"]] = dxp
        dxs = self._a2a(dxr, ctx["recv"], ctx["send"])                 # send order
        dhn2 = moe.combine(dxs, ctx["pos"], None)
        return dhn2, dw


class FusedExpertParallel(ExpertParallel):
    """Expert parallelism on the symmetric peer-memory heap (path d), with no
    host synchronisation.

    Plan: per-expert counts (a scatter-add on the device) are all-gathered
    with NCCL straight into a device buffer; one kernel turns them into every
    local pair's owner rank and row in the owner's receive buffer (expert-major,
    each expert padded to 64 rows, source ranks in rank order), and the owner's
    padded expert offsets and grouped-GEMM tile table. Nothing returns to the
    host; a receive buffer that is too small sets a device flag that
    ``check_overflow`` reads once per optimizer step.

    Dispatch, two forms. ``dispatch="push"`` (the default, measured faster):
    every rank stores its token rows straight into the owners' receive
    buffers with P2P stores, then a barrier, a pad-zeroing pass and the
    grouped GEMM. ``dispatch="pull"``: every rank copies its token
    rows into its heap token buffer and pushes one 4-byte index entry per
    (token, expert) pair into the owner's heap index (which rank, which
    token row, at the pair's receive row); after one device barrier the
    owner's gate/up grouped GEMM stages the receive buffer itself in its
    prologue: each CTA pulls 64-row groups from the peers' token buffers over
    NVLink (pad rows zero-filled), publishes a per-group flag, and the tiles
    start as soon as their groups are in, so each token row crosses NVLink
    once, inside the GEMM launch. On B200 the pull form measured slower than
    push + GEMM (the in-kernel copy warps slow the tiles more than a separate
    full-occupancy copy pass costs), so it is kept as an option. Combine:
    each source rank pulls its pairs' expert outputs from the owners' heaps and
    reduces them with the routing weights and the residual in the same kernel.
    Backward: the expert side is recomputed from the saved token rows (one more
    dispatch and gate/up GEMM) instead of keeping receive-buffer-sized
    activations per layer; w * dy rows are pushed to the owners, the routing
    gradient's dot products and the input gradients are pulled back. Device
    barriers (epoch flags) order the phases.
    """

    def __init__(self, ctx, cfg, lo, hi, heap, cap_rows: int, dispatch: str = "push"):
        super().__init__(ctx, cfg, lo, hi)
        if dispatch not in ("pull", "push"):
            raise ValueError("dispatch must be pull|push")
        H = cfg.hidden_size
        I = cfg.moe_intermediate_size
        self.heap = heap
        self.cap = int(cap_rows) // 64 * 64
        self.o_recv, self.recv = heap.alloc(self.cap * H)
        self.o_y, self.ybuf = heap.alloc(self.cap * H)
        self.o_dy, self.dybuf = heap.alloc(self.cap * H)
        self.o_dx, self.dxbuf = heap.alloc(self.cap * H)
        self.H, self.I = H, I
        self.overflow = torch.zeros(1, dtype=torch.int32, device=ctx.device)
        self.dispatch = dispatch
        if dispatch == "pull":
            self.tok_rows = max(1, self.cap // max(1, cfg.num_experts_per_tok))
            self.o_tok, self.tok = heap.alloc(self.tok_rows * H)
            self.o_index, self.index = heap.alloc(self.cap, dtype=torch.int32)
            self.tok_peers = ops.native().symm_peer_addrs(heap.id, self.o_tok)
            self.flags = torch.zeros(self.cap // 64, dtype=torch.int32, device=ctx.device)
            self._stage_epoch = 0

    @staticmethod
    def heap_bytes(cfg, cap_rows: int, dispatch: str = "push") -> int:
        """Symmetric-heap bytes the buffers of ``cap_rows`` receive rows need."""
        cap = int(cap_rows) // 64 * 64
        H = cfg.hidden_size
        n = 4 * cap * H * 2 + 4 * 256
        if dispatch == "pull":
            n += max(1, cap // max(1, cfg.num_experts_per_tok)) * H * 2 + cap * 4 + 2 * 256
        return n

    def _plan(self, idx):
        T, k = idx.shape
        dev = idx.device
        flat = idx.reshape(-1).long()
        counts = torch.zeros(self.E, dtype=torch.int32, device=dev)
        counts.scatter_add_(0, flat, torch.ones_like(flat, dtype=torch.int32))
        allc = torch.empty(self.W * self.E, dtype=torch.int32, device=dev)
        dist.all_gather_into_tensor(allc, counts, group=self.ctx.group)
        dst_rank = torch.empty(T * k, dtype=torch.int32, device=dev)
        dst_row = torch.empty(T * k, dtype=torch.long, device=dev)
        offs = torch.empty(self.El + 1, dtype=torch.int32, device=dev)
        tot = torch.empty(self.El, dtype=torch.int32, device=dev)
        ncap = self.cap // 128 + self.El
        tiles = torch.zeros(ncap * 4, dtype=torch.int32, device=dev)
        ntiles = torch.zeros(1, dtype=torch.int32, device=dev)
        ops.native().moe_ep_plan(idx.int().contiguous(), allc, self.W, self.ctx.rank, self.cap, dst_rank, dst_row,
                                 offs, tot, tiles, ntiles, self.overflow)
        return dict(dst_rank=dst_rank, dst_row=dst_row,
                    plan=moe.Plan(None, None, offs, tiles, ntiles, tot, self.cap))

    def check_overflow(self) -> None:
        if int(self.overflow.item()):
            self.overflow.zero_()
            raise RuntimeError("expert-parallel receive buffer overflow: raise ep_capacity")

    def _dispatch_and_up(self, W, hn2, pl):
        """Rows to the owners, pad rows zeroed, gate/up GEMM on the receive buffer."""
        if self.dispatch == "pull" and hn2.shape[0] <= self.tok_rows:
            return self._pull_and_up(W, hn2, pl)
        C = ops.native()
        T, k = pl["dst_rank"].numel() // self.k, self.k
        src_row = torch.arange(T * k, device=hn2.device) // k
        C.symm_ep_scatter(self.heap.id, self.o_recv, hn2, src_row, pl["dst_rank"], pl["dst_row"], None, self.cap)
        self.heap.barrier()                                   # all rows delivered
        xp = self.recv[: self.cap * self.H].view(self.cap, self.H)
        C.moe_zero_pad_rows(xp, pl["plan"].offsets, pl["plan"].counts, self.H)
        gu = moe.plan_mm(xp, W["experts_gate_up"], pl["plan"])
        return xp, gu

    def _pull_and_up(self, W, hn2, pl):
        """Pull dispatch: index entries to the owners, then the gate/up grouped
        GEMM that stages its own receive rows from the peers' token buffers."""
        C = ops.native()
        T, H = hn2.shape
        self.tok[: T * H].view(T, H).copy_(hn2)
        C.symm_ep_index_push(self.heap.id, self.o_index, pl["dst_rank"], pl["dst_row"], self.k, self.cap)
        plan = pl["plan"]
        C.moe_index_pads(self.index, plan.offsets, plan.counts)
        self.heap.barrier()                                   # every rank's token rows and index entries are in
        xp = self.recv[: self.cap * H].view(self.cap, H)
        wgu = W["experts_gate_up"]
        gu = torch.empty(self.cap, wgu.shape[1], dtype=hn2.dtype, device=hn2.device)
        self._stage_epoch += 1
        C.gemm_grouped_dev_pull(xp, wgu, gu, plan.tiles, plan.ntiles, self.tok_peers, H, self.index,
                                plan.offsets[-1:], self.flags, self._stage_epoch, False)
        return xp, gu

    def forward(self, eng, W, hn2, x2, probs, idx, wts):
        T, k = idx.shape
        self.k = k
        pl = self._plan(idx)
        xp, gu = self._dispatch_and_up(W, hn2, pl)
        a = ops.swiglu_fwd(gu)
        yp = self.ybuf[: self.cap * self.H].view(self.cap, self.H)
        moe.plan_mm(a, W["experts_down"], pl["plan"], out=yp)
        del gu, a
        self.heap.barrier()                                   # expert outputs ready
        y = torch.empty_like(x2)
        ops.native().symm_ep_gather(self.heap.id, self.o_y, pl["dst_rank"].view(T, k), pl["dst_row"].view(T, k),
                                    wts.float().contiguous(), x2, y, None, None, self.H)
        self.heap.barrier()                                   # pulls done before ybuf is reused
        ctx = dict(probs=probs, idx=idx, wts=wts, fused=True, hn2=hn2, **pl)
        return y, ctx

    def backward(self, eng, W, G, ctx, dx3):
        if not ctx.get("fused"):
            return super().backward(eng, W, G, ctx, dx3)
        C = ops.native()
        T, k = ctx["idx"].shape
        H = self.H
        dev = dx3.device
        pl = ctx["plan"]
        # recompute the expert side: dispatch, gate/up, SwiGLU, down (y is needed for the routing gradient)
        xp, gu = self._dispatch_and_up(W, ctx["hn2"], ctx)
        a = ops.swiglu_fwd(gu)
        yp = self.ybuf[: self.cap * H].view(self.cap, H)
        moe.plan_mm(a, W["experts_down"], pl, out=yp)
        self.heap.barrier()                                   # expert outputs ready for the pulls
        dw = torch.empty(T, k, dtype=torch.float32, device=dev)
        C.symm_ep_gather(self.heap.id, self.o_y, ctx["dst_rank"].view(T, k), ctx["dst_row"].view(T, k), None, None,
                         dx3, dx3, dw, H)
        src_row = torch.arange(T * k, device=dev) // k
        C.symm_ep_scatter(self.heap.id, self.o_dy, dx3, src_row, ctx["dst_rank"], ctx["dst_row"],
                          ctx["wts"].reshape(-1).float().contiguous(), self.cap)
        self.heap.barrier()                                   # w * dy rows delivered; y reads done
        dyp = self.dybuf[: self.cap * H].view(self.cap, H)
        C.moe_zero_pad_rows(dyp, pl.offsets, pl.counts, H)
        da = moe.plan_mm(dyp, W["experts_down"], pl, w_t=False)
        eng._plan_wgrad(G["experts_down"], dyp, a, pl)
        dgu = ops.swiglu_bwd(da, gu, gu)
        del da
        dxp = self.dxbuf[: self.cap * H].view(self.cap, H)
        moe.plan_mm(dgu, W["experts_gate_up"], pl, w_t=False, out=dxp)
        eng._plan_wgrad(G["experts_gate_up"], dgu, xp, pl)
        self.heap.barrier()                                   # input grads ready
        dhn2 = torch.empty(T, H, dtype=dx3.dtype, device=dev)
        C.symm_ep_gather(self.heap.id, self.o_dx, ctx["dst_rank"].view(T, k), ctx["dst_row"].view(T, k), None, None,
                         dhn2, None, None, H)
        self.heap.barrier()                                   # pulls done before buffers are reused
        return dhn2, dw
