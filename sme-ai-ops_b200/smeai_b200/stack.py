"""Llama-2-7B-shape Q2_K linear stack (the decode/prefill benchmark workload).

Per layer, with the inputs of every linear re-quantized to Q8_K (rmsnorm
includes the layer's norm weight, as sme_ai_rmsnorm_f32 and llama's
attn_norm / ffn_norm / output_norm do):
    xq  = Q8_K(rmsnorm(x) * attn_norm)
    qkv = [Wq; Wk; Wv] xq                       (one fused GEMV, 3 x 4096 rows)
    v   = qkv[v]   -- attention over a single position returns v itself, so
                      the attention math is skipped without changing shapes
    x   = x + Wo Q8_K(v)                        (residual fused in the epilogue)
    h   = silu(Wg xq') * (Wu xq'),  xq' = Q8_K(rmsnorm(x) * ffn_norm)
                                                (gate/up rows interleaved, one GEMV
                                                 with the silu*mul epilogue)
    x   = x + Wd Q8_K(h)
then logits = Wlm Q8_K(rmsnorm(x) * output_norm).

Multi-GPU: every weight is row-sharded over the ranks (32-row aligned slices
of each of Wq/Wk/Wv/Wo/Wg/Wu/Wd/Wlm); activations are replicated and each
linear's output slices are all-gathered over NCCL.  Weights are drawn from a
seeded N(0, std) per full matrix and sliced, so every world size computes the
same model.
"""
from __future__ import annotations

import math

import torch

from . import EPI_RESIDUAL, EPI_SILU_MUL, EPI_STORE, Q2K_BLOCK_BYTES, Q8K_BLOCK_BYTES, QK_K
from . import q2k as Q

LLAMA7B = dict(n_layers=32, hidden=4096, ffn=11008, vocab=32000)


def shard_range(n: int, rank: int, world: int, align: int = 32):
    """Contiguous row slice [lo, hi) of rank `rank`: every slice but the last is
    ceil(n / world / align) * align rows (the last may be shorter or empty)."""
    per = shard_stride(n, world, align)
    lo = min(n, rank * per)
    hi = min(n, lo + per)
    return lo, hi


def shard_stride(n: int, world: int, align: int = 32) -> int:
    return int(math.ceil(n / world / align)) * align


def token_range(n: int, rank: int, world: int):
    """Tokens [lo, hi) of rank `rank` when the tokens of a prefill are split
    over `world` ranks (sequence sharding): sizes differ by at most one."""
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_rows(full, local, n: int, world: int, group=None, scratch=None):
    """full[:, :n] <- the ranks' row slices in rank order (torch.distributed).

    `local` is this rank's [B, hi-lo] slice; slices follow shard_range(n, ., world).
    When every slice has the same length and B == 1 the gather lands in `full`
    directly; otherwise the slices are padded to the common stride, gathered into
    `scratch` ([world * B, stride], allocated if None) and copied out."""
    import torch.distributed as dist
    B, have = local.shape
    stride = shard_stride(n, world)
    if B == 1 and stride * world == n and have == stride and full.is_contiguous():
        dist.all_gather_into_tensor(full.view(-1)[:n], local.reshape(-1), group=group)
        return full
    if scratch is None:
        scratch = local.new_empty((world * B, stride))
    send = local.new_zeros((B, stride))
    send[:, :have].copy_(local)
    dist.all_gather_into_tensor(scratch, send, group=group)
    full[:, :n].copy_(scratch.view(world, B, stride).permute(1, 0, 2).reshape(B, world * stride)[:, :n])
    return full


def gemv_bytes(rows: int, k: int, cols: int, out_rows: int | None = None) -> int:
    """Algorithmic bytes of one Q2_K GEMV: weights + Q8_K activations + fp32 out."""
    nb = k // QK_K
    out_rows = rows if out_rows is None else out_rows
    return rows * nb * Q2K_BLOCK_BYTES + cols * nb * Q8K_BLOCK_BYTES + cols * out_rows * 4


class Q2KDecodeStack:
    def __init__(self, n_layers=32, hidden=4096, ffn=11008, vocab=32000, batch=1, rank=0, world=1,
                 device=None, seed=0, std=0.02, eps=1e-5, group=None, keep_blocks=False, quant="separate",
                 norm_weights=True, tokens=None):
        # tokens=(lo, hi): this stack runs tokens lo..hi-1 of a batch of `batch`
        # (sequence sharding of a prefill: every rank holds the full weights
        # and its own tokens; rows of x0 are those of the whole batch's draw)
        self.batch_global = batch
        self.tok_lo, self.tok_hi = (0, batch) if tokens is None else (int(tokens[0]), int(tokens[1]))
        assert 0 <= self.tok_lo < self.tok_hi <= batch, (tokens, batch)
        batch = self.tok_hi - self.tok_lo
        self.L, self.H, self.F, self.V = n_layers, hidden, ffn, vocab
        self.B, self.rank, self.world, self.eps, self.group = batch, rank, world, eps, group
        # where each linear's input is quantized to Q8_K: "fused" = inside the
        # GEMV's prologue; "separate" = a quantizer kernel before the GEMV;
        # "mixed" = fused where an RMSNorm comes first (qkv, gate/up, lm_head),
        # separate for the plain re-quantizations (o, down).  All three give
        # bit-identical results.  "program" (one GPU; batch 1, 2, 4 or 8): the
        # whole step is ONE persistent kernel (Q2KProgram) -- same bits again.
        # "peer" (N > 1 GPUs; batch 1, 2, 4 or 8): every GEMV stores its rows into
        # all ranks' copies of the next input and signals them in the same kernel
        # (the all-gather fused in, over CUDA-IPC peer memory); the next GEMV waits
        # for every rank's rows.  Falls back to "separate" + NCCL when a shard is
        # not 32-row aligned or the peers cannot be mapped.  "tc" (prefill, any
        # batch): every linear on the tensor-core GEMM with the same epilogues,
        # the quantizers as separate kernels -- same bits as the GEMV placements;
        # on N GPUs its slices are all-gathered over NCCL.
        # "mgprog" (N GPUs, or one GPU to check the wiring; batch 1, 2, 4 or 8):
        # the whole step as ONE persistent kernel per rank over its row shards,
        # every finished row stored into every rank's copy of the phase's
        # output in the same kernel (Q2KMGProgram) -- the default on N > 1.
        assert quant in ("fused", "separate", "mixed", "program", "peer", "tc", "mgprog")
        if quant in ("program", "peer", "mgprog") and world > 1:
            aligned = all((shard_range(n, q, world)[1] - shard_range(n, q, world)[0]) % 32 == 0
                          for n in (hidden, ffn, vocab) for q in range(world - 1))
            if not (aligned and batch in (1, 2, 4, 8)):
                quant = "separate"
            elif quant == "program":
                quant = "mgprog"
        elif quant == "peer":
            quant = "program"
        if quant in ("program", "mgprog") and batch not in (1, 2, 4, 8):
            quant = "separate"
        self.prog = None
        self.quant = quant
        self.dev = device or torch.device("cuda", torch.cuda.current_device())
        assert hidden % QK_K == 0 and ffn % QK_K == 0
        self.h_lo, self.h_hi = shard_range(hidden, rank, world)
        self.f_lo, self.f_hi = shard_range(ffn, rank, world)
        self.v_lo, self.v_hi = shard_range(vocab, rank, world)
        hs, fs, vs = self.h_hi - self.h_lo, self.f_hi - self.f_lo, self.v_hi - self.v_lo
        self.hs, self.fs, self.vs = hs, fs, vs
        self.layers = []
        self.blocks = [] if keep_blocks else None   # raw ggml blocks per layer (tests)
        self.weight_bytes = 0
        for li in range(n_layers):
            wq, wk, wv = (self._draw(seed, li, m, hidden, hidden, self.h_lo, self.h_hi, std) for m in range(3))
            wqkv = Q.Q2KMatrix(torch.cat([wq, wk, wv], 0), 3 * hs, hidden)
            wo_b = self._draw(seed, li, 3, hidden, hidden, self.h_lo, self.h_hi, std)
            wo = Q.Q2KMatrix(wo_b, hs, hidden)
            wg = self._draw(seed, li, 4, ffn, hidden, self.f_lo, self.f_hi, std)
            wu = self._draw(seed, li, 5, ffn, hidden, self.f_lo, self.f_hi, std)
            wgu = Q.Q2KMatrix(torch.stack([wg, wu], 1).reshape(2 * fs, -1), 2 * fs, hidden)
            wd_b = self._draw(seed, li, 6, hidden, ffn, self.h_lo, self.h_hi, std)
            wd = Q.Q2KMatrix(wd_b, hs, ffn)
            if keep_blocks:
                self.blocks.append(dict(q=wq, k=wk, v=wv, o=wo_b, g=wg, u=wu, d=wd_b))
            del wq, wk, wv, wg, wu
            self.layers.append((wqkv, wo, wgu, wd))
            self.weight_bytes += wqkv.n_rows * wqkv.nb * 84 + wo.n_rows * wo.nb * 84 + \
                wgu.n_rows * wgu.nb * 84 + wd.n_rows * wd.nb * 84
        # RMSNorm weights (attn_norm, ffn_norm per layer, output_norm): seeded
        # draws around 1, replicated on every rank; None = no weight
        self.attn_norm, self.ffn_norm, self.out_norm = [None] * n_layers, [None] * n_layers, None
        if norm_weights:
            gn = torch.Generator(device=self.dev).manual_seed(seed * 7919 + 31)
            nw = lambda: 1.0 + 0.1 * torch.randn(hidden, generator=gn, device=self.dev)
            self.attn_norm = [nw() for _ in range(n_layers)]
            self.ffn_norm = [nw() for _ in range(n_layers)]
            self.out_norm = nw()
        lm_b = self._draw(seed, n_layers, 7, vocab, hidden, self.v_lo, self.v_hi, std)
        self.lm = Q.Q2KMatrix(lm_b, vs, hidden)
        self.lm_blocks = lm_b if keep_blocks else None
        self.weight_bytes += self.lm.n_rows * self.lm.nb * 84
        torch.cuda.synchronize()
        B, d, f32, u8 = batch, self.dev, torch.float32, torch.uint8
        self.x0 = torch.randn((self.batch_global, hidden), generator=torch.Generator(device=d).manual_seed(seed + 12345),
                              device=d, dtype=f32)[self.tok_lo:self.tok_hi].contiguous()
        self.x = torch.empty_like(self.x0)
        self.xq = torch.empty((B, hidden // QK_K * Q8K_BLOCK_BYTES), dtype=u8, device=d)
        self.qkv = torch.empty((B, 3 * hs), dtype=f32, device=d)
        self.v_full = torch.empty((B, hidden), dtype=f32, device=d)
        self.vq = torch.empty_like(self.xq)
        self.x_loc = torch.empty((B, hs), dtype=f32, device=d)
        self.h_loc = torch.empty((B, fs), dtype=f32, device=d)
        self.h_full = torch.empty((B, ffn), dtype=f32, device=d)
        self.hq = torch.empty((B, ffn // QK_K * Q8K_BLOCK_BYTES), dtype=u8, device=d)
        self.lg_loc = torch.empty((B, vs), dtype=f32, device=d)
        self.logits = torch.empty((B, vocab), dtype=f32, device=d)
        self.x_loc_d = torch.empty((B, hs), dtype=f32, device=d)   # the down phase's local rows (mgprog)
        self.arena = None
        if self.quant == "peer":
            self._setup_peer()

    # --------------------------------------------------------------- weights
    def _draw(self, seed, layer, mat, rows, k, lo, hi, std):
        g = torch.Generator(device=self.dev).manual_seed(seed * 1_000_003 + layer * 16 + mat)
        # draw the full matrix in row chunks with one generator: identical for every world size
        out = None
        chunk = max(1, (1 << 27) // k)
        for r0 in range(0, rows, chunk):
            r1 = min(rows, r0 + chunk)
            w = torch.randn((r1 - r0, k), generator=g, device=self.dev) * std
            a, b = max(lo, r0), min(hi, r1)
            if a < b:
                part = Q.quantize_q2k(w[a - r0:b - r0])
                out = part if out is None else torch.cat([out, part], 0)
        return out

    # --------------------------------------------------------------- collectives
    def _gather(self, full: torch.Tensor, local: torch.Tensor, lo: int, hi: int):
        """full[:, :] <- concatenation over ranks of local (row slices)."""
        if self.world == 1:
            if full.data_ptr() != local.data_ptr():
                full.copy_(local)
            return
        gather_rows(full, local, full.shape[1], self.world, self.group)

    # --------------------------------------------------------------- fused exchange
    def _setup_peer(self):
        """Peer arena and the exchange descriptors of every GEMV ("peer" mode)."""
        from .peer import PeerArena, PeerUnavailable, decode_plan, make_exchange
        B, H, F, V, L, W, r = self.B, self.H, self.F, self.V, self.L, self.world, self.rank
        layout = [("x", B * H * 4), ("v", B * H * 4), ("h", B * F * 4), ("lg", B * V * 4), ("sig", (4 * L + 1) * 4),
                  ("epoch", 4)]
        try:
            ar = PeerArena(layout, self.dev, r, W, self.group)
        except PeerUnavailable:
            self.quant = "separate"
            return
        self.arena = ar
        f32 = torch.float32
        self.x, self.v_full = ar.tensor("x", f32, (B, H)), ar.tensor("v", f32, (B, H))
        self.h_full, self.logits = ar.tensor("h", f32, (B, F)), ar.tensor("lg", f32, (B, V))
        epoch = ar.addr(r, "epoch")
        exs = []
        for name, dst, ld, row0, sig, wait, count in decode_plan(H, F, V, L, r, W, shard_range):
            if name == "end":
                self.end = (ar.addr(r, "sig", 4 * wait), count, epoch)
                continue
            exs.append(make_exchange([ar.addr(q, buf, 4 * off) for q, buf, off in dst], ld, row0,
                                     [ar.addr(q, "sig", 4 * sig) for q in range(W)],
                                     ar.addr(r, "sig", 4 * wait) if wait is not None else 0,
                                     count if wait is not None else 0, epoch if wait is not None else 0))
        self.ex = [tuple(exs[4 * li:4 * li + 4]) for li in range(L)]
        self.ex_lm = exs[4 * L]

    def _step_peer(self):
        from . import check, lib
        B, e = self.B, self.eps
        xs = self.x[:, self.h_lo:self.h_hi]
        for li, ((wqkv, wo, wgu, wd), (eq, eo, egu, ed)) in enumerate(zip(self.layers, self.ex)):
            wqkv.mul_mat_f32_peer(self.x, B, self.qkv, eq, rms_eps=e, norm_w=self.attn_norm[li])
            wo.mul_mat_f32_peer(self.v_full, B, xs, eo, EPI_RESIDUAL, resid=xs)
            wgu.mul_mat_f32_peer(self.x, B, self.h_full[:, self.f_lo:self.f_hi], egu, EPI_SILU_MUL, rms_eps=e,
                                 norm_w=self.ffn_norm[li])
            wd.mul_mat_f32_peer(self.h_full, B, xs, ed, EPI_RESIDUAL, resid=xs)
        self.lm.mul_mat_f32_peer(self.x, B, self.logits[:, self.v_lo:self.v_hi], self.ex_lm, rms_eps=e,
                                 norm_w=self.out_norm)
        sig, count, epoch = self.end
        check(lib().smeai_peer_step_end(sig, count, epoch, Q.cur_stream()), "peer_step_end")
        return self.logits

    # --------------------------------------------------------------- one token
    def _lin(self, m, x, out, epilogue=EPI_STORE, resid=None, rms=False, qbuf=None, norm_w=None):
        """One linear: y = W Q8_K([rmsnorm * norm_w] x) with the stack's quantization placement."""
        fused = self.quant == "fused" or (self.quant == "mixed" and rms)
        if self.quant == "tc":
            if rms:
                Q.rms_quantize_q8k(x, self.eps, out=qbuf, norm_w=norm_w)
            else:
                Q.quantize_q8k(x, out=qbuf)
            m.mul_mat_tc(qbuf, self.B, out=out, epilogue=epilogue, resid=resid)
        elif fused:
            m.mul_mat_f32_ex(x, self.B, out=out, epilogue=epilogue, resid=resid,
                             rms_eps=self.eps if rms else None, norm_w=norm_w if rms else None)
        else:
            if rms:
                Q.rms_quantize_q8k(x, self.eps, out=qbuf, norm_w=norm_w)
            else:
                Q.quantize_q8k(x, out=qbuf)
            m.mul_mat(qbuf, self.B, out=out, epilogue=epilogue, resid=resid)

    def step(self, x_in: torch.Tensor | None = None):
        """Enqueue one pass of the stack on the current stream; returns logits."""
        B, H, hs = self.B, self.H, self.hs
        self.x.copy_(self.x0 if x_in is None else x_in)
        one = self.world == 1
        if self.quant == "program":
            if self.prog is None:
                self.prog = self._build_program()
            self.prog.run()
            return self.logits
        if self.quant == "mgprog":
            if self.prog is None:
                self.prog = self._build_mg_program()
            self.prog.run()
            self.prog.gather(4 * self.L, self.logits)
            return self.logits
        if self.quant == "peer":
            return self._step_peer()
        L = self._lin
        for li, (wqkv, wo, wgu, wd) in enumerate(self.layers):
            an, fn = self.attn_norm[li], self.ffn_norm[li]
            L(wqkv, self.x, self.qkv, rms=True, qbuf=self.xq, norm_w=an)
            v_loc = self.qkv[:, 2 * hs:3 * hs]
            if one:
                L(wo, v_loc, self.x, EPI_RESIDUAL, self.x, qbuf=self.vq)
                L(wgu, self.x, self.h_full, EPI_SILU_MUL, rms=True, qbuf=self.xq, norm_w=fn)
                L(wd, self.h_full, self.x, EPI_RESIDUAL, self.x, qbuf=self.hq)
            else:
                self._gather(self.v_full, v_loc.contiguous(), self.h_lo, self.h_hi)
                L(wo, self.v_full, self.x_loc, EPI_RESIDUAL, self.x[:, self.h_lo:self.h_hi], qbuf=self.vq)
                self._gather(self.x, self.x_loc, self.h_lo, self.h_hi)
                L(wgu, self.x, self.h_loc, EPI_SILU_MUL, rms=True, qbuf=self.xq, norm_w=fn)
                self._gather(self.h_full, self.h_loc, self.f_lo, self.f_hi)
                L(wd, self.h_full, self.x_loc, EPI_RESIDUAL, self.x[:, self.h_lo:self.h_hi], qbuf=self.hq)
                self._gather(self.x, self.x_loc, self.h_lo, self.h_hi)
        if one:
            L(self.lm, self.x, self.logits, rms=True, qbuf=self.xq, norm_w=self.out_norm)
        else:
            L(self.lm, self.x, self.lg_loc, rms=True, qbuf=self.xq, norm_w=self.out_norm)
            self._gather(self.logits, self.lg_loc, self.v_lo, self.v_hi)
        return self.logits

    def _build_program(self):
        from . import IN_F32, IN_F32_RMS
        hs = self.hs
        phases = []
        for li, (wqkv, wo, wgu, wd) in enumerate(self.layers):
            phases += [
                dict(w=wqkv, x=self.x, input=IN_F32_RMS, y=self.qkv, norm_w=self.attn_norm[li]),
                dict(w=wo, x=self.qkv[:, 2 * hs:3 * hs], input=IN_F32, y=self.x, epilogue=EPI_RESIDUAL,
                     resid=self.x),
                dict(w=wgu, x=self.x, input=IN_F32_RMS, y=self.h_full, epilogue=EPI_SILU_MUL,
                     norm_w=self.ffn_norm[li]),
                dict(w=wd, x=self.h_full, input=IN_F32, y=self.x, epilogue=EPI_RESIDUAL, resid=self.x),
            ]
        phases.append(dict(w=self.lm, x=self.x, input=IN_F32_RMS, y=self.logits, norm_w=self.out_norm))
        return Q.Q2KProgram(phases, self.B, rms_eps=self.eps)

    def _build_mg_program(self):
        """The step as one kernel per rank over the rank's row shards; every
        phase names the phase it reads (global rows) explicitly."""
        from . import IN_F32, IN_F32_RMS
        H, F, V, hs = self.H, self.F, self.V, self.hs
        phases = []
        for li, (wqkv, wo, wgu, wd) in enumerate(self.layers):
            b = 4 * li
            x_in = dict(x_src=b - 1) if li else dict(x=self.x)
            resid_in = dict(resid_src=b - 1, resid_row0=self.h_lo) if li else \
                dict(resid=self.x, resid_row0=self.h_lo)
            phases += [
                dict(w=wqkv, input=IN_F32_RMS, norm_w=self.attn_norm[li], out_rows=H, ex_lo=2 * hs, ex_hi=3 * hs,
                     ex_row0=self.h_lo, y=self.qkv, **x_in),
                dict(w=wo, input=IN_F32, x_src=b, epilogue=EPI_RESIDUAL, out_rows=H, ex_hi=hs, ex_row0=self.h_lo,
                     y=self.x_loc, **resid_in),
                dict(w=wgu, input=IN_F32_RMS, x_src=b + 1, norm_w=self.ffn_norm[li], epilogue=EPI_SILU_MUL,
                     out_rows=F, ex_hi=self.fs, ex_row0=self.f_lo, y=self.h_loc),
                dict(w=wd, input=IN_F32, x_src=b + 2, epilogue=EPI_RESIDUAL, resid_src=b + 1, resid_row0=self.h_lo,
                     out_rows=H, ex_hi=hs, ex_row0=self.h_lo, y=self.x_loc_d),
            ]
        phases.append(dict(w=self.lm, input=IN_F32_RMS, x_src=4 * self.L - 1, norm_w=self.out_norm, out_rows=V,
                           ex_hi=self.vs, ex_row0=self.v_lo, y=self.lg_loc))
        return Q.Q2KMGProgram(phases, self.B, self.rank, self.world, rms_eps=self.eps, group=self.group)

    # --------------------------------------------------------------- accounting
    def ops_per_step(self) -> int:
        """Integer multiply-adds x 2 of every linear in a step on this rank
        (the tensor-core roofline's unit)."""
        return sum(2 * self.B * m.n_rows * m.k for _, m in self.gemv_list())

    def launches_per_step(self) -> int:
        """Kernels of this library per step: one GEMV per linear (the batch is
        split into launches of 8, 4, 2, 1 tokens) plus one quantizer per
        linear whose quantization is not fused."""
        if self.quant == "program":
            return 1
        if self.quant == "mgprog":
            return 2                       # the program and the gather of the logits
        if self.quant == "peer":
            return self.L * 4 + 2          # the GEMVs and the step-end kernel
        if self.quant == "tc":             # per linear: quantizer, operand prepass, GEMM
            return (self.L * 4 + 1) * 3
        chunks = self.B // 8 + bin(self.B % 8).count("1")
        per_layer = {"fused": 0, "separate": 4, "mixed": 2}[self.quant]
        return (self.L * 4 + 1) * chunks + self.L * per_layer + (1 if self.quant == "separate" else 0)

    def gemv_list(self):
        """(name, matrix, k, cols, out_rows) of every GEMV in a step."""
        out = []
        for wqkv, wo, wgu, wd in self.layers:
            out += [("qkv", wqkv), ("o", wo), ("gate_up", wgu), ("down", wd)]
        out.append(("lm_head", self.lm))
        return out

    def algorithmic_bytes(self) -> int:
        """Bytes one step must move on this rank: every GEMV's weights, Q8_K
        inputs and fp32 outputs (the quantizers' few KB are not counted)."""
        tot = 0
        for name, m in self.gemv_list():
            out_rows = m.n_rows // 2 if name == "gate_up" else m.n_rows
            tot += gemv_bytes(m.n_rows, m.k, self.B, out_rows)
        return tot

    def free(self):
        if self.prog is not None:
            self.prog.free()
            self.prog = None
        if self.arena is not None:
            # no rank may still store into this arena: all ranks' steps are done
            torch.cuda.synchronize(self.dev)
            import torch.distributed as dist
            dist.barrier(group=self.group)
            self.x = self.v_full = self.h_full = self.logits = None
            self.arena.close()
            self.arena = None
        for layer in self.layers:
            for m in layer:
                m.free()
        self.lm.free()
