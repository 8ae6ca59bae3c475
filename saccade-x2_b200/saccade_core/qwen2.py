"""Qwen2 decoder with every linear a C-TARQ op, on the GPU (saccade-runner/src/model.rs).

    Qwen2Config            model.rs's Qwen2Config (hidden, intermediate, layers, heads, ...)
    random_checkpoint      a random-init model in the reference's compiled format: every projection
                           packed by the GPU packer (compress.rs:6-176, bit-identical to the
                           reference's), thresholds calibrated per projection (calibration.rs:10-47)
    Qwen2Model             Qwen2Model::forward (model.rs:508-523) on one GPU or one tensor-parallel rank:
                           embedding, per layer input RMSNorm -> q/k/v (one grouped C-TARQ launch,
                           biases after the f16 rounding) -> RoPE -> KV cache -> GQA attention -> o
                           -> residual -> RMSNorm -> gate/up (one launch) -> SiLU * up -> down ->
                           residual; final RMSNorm and lm_head; greedy decoding (verify.rs:98-130).

Precision follows the reference: f32 everywhere except the f16 inputs and outputs of the C-TARQ
ops (the projection layer's casts, model.rs:52-64); the KV cache is f32.  The embedding / lm_head
table holds f16 values (a random init drawn and rounded to f16, held in f32 by the reference), so
lm_head runs as two f16 GEMMs with f32 accumulation on an exact hi/lo f16 split of the f32 hidden
state (x = hi + lo to 2^-22 relative).

Tensor parallelism (tp = (rank, world, group)): q/k/v and gate/up keep this rank's output rows
(whole heads; a KV head shared by two ranks when there are fewer KV heads than ranks), o and down
keep the matching input columns.  A row-sharded layer sees only its slice of each token, so it
writes one f32 exchange buffer [y_base | y_delta | router sums] (sc_forward_split), the buffers are
summed over the group by one NCCL all-reduce, and sc_finalize_split routes every token on the
summed sums and rounds.  The lm_head is vocab-parallel: each rank scores its slice of the
vocabulary and greedy decoding all-gathers each rank's (max, argmax) per sequence.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from . import _lib
from ._lib import LIB, check
from .compress import ProfileRunner, compress_tensor_to_saccade, compute_percentile_threshold
from .graph import no_gc
from .op import GroupRouting, SaccadeConfig, SaccadeLinearGroup, SaccadeLinearOp, SparseDeltaMatrix, flush_deferred

PROJ = ("q", "k", "v", "o", "gate", "up", "down")


@dataclass
class Qwen2Config:
    hidden: int
    intermediate: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    rope_theta: float = 1.0e6
    eps: float = 1.0e-6
    tie_embeddings: bool = True

    @staticmethod
    def qwen2_0_5b(layers: int = 24) -> "Qwen2Config":
        return Qwen2Config(896, 4864, layers, 14, 2, 64, 151936, tie_embeddings=True)

    @staticmethod
    def qwen2_7b(layers: int = 28) -> "Qwen2Config":
        return Qwen2Config(3584, 18944, layers, 28, 4, 128, 152064, tie_embeddings=False)

    @staticmethod
    def qwen2_72b(layers: int = 80) -> "Qwen2Config":
        return Qwen2Config(8192, 29568, layers, 64, 8, 128, 152064, tie_embeddings=False)

    def proj_shape(self, name: str):
        """(out_features, in_features) of a projection."""
        qd, kvd = self.heads * self.head_dim, self.kv_heads * self.head_dim
        return {"q": (qd, self.hidden), "k": (kvd, self.hidden), "v": (kvd, self.hidden), "o": (self.hidden, qd),
                "gate": (self.intermediate, self.hidden), "up": (self.intermediate, self.hidden),
                "down": (self.hidden, self.intermediate)}[name]


def rope_tables(cfg: Qwen2Config, max_pos: int):
    """RotaryEmbedding::new (model.rs:111-132) in f32: inv_freq_i = 1 / theta^(2i / hd), angle = t * inv_freq,
    the angles duplicated over both halves of the head."""
    hd = cfg.head_dim
    theta = np.float32(cfg.rope_theta)
    inv = np.array([np.float32(1.0) / np.power(theta, np.float32(i) / np.float32(hd), dtype=np.float32)
                     for i in range(0, hd, 2)], dtype=np.float32)
    t = np.arange(max_pos, dtype=np.float32).reshape(-1, 1)
    freqs = (t * inv.reshape(1, -1)).astype(np.float32)
    full = np.concatenate([freqs, freqs], axis=1)
    return np.cos(full).astype(np.float32), np.sin(full).astype(np.float32)


# ------------------------------------------------------------------ tensor-parallel layout

def head_split(cfg: Qwen2Config, rank: int, world: int):
    """This rank's query heads [q0, q1) and KV heads [k0, k1).  With at least as many KV heads as
    ranks, each rank takes whole KV groups; with fewer, `world / kv_heads` ranks share a KV head (each
    computes it) and split its query heads as evenly as possible."""
    G = cfg.heads // cfg.kv_heads
    if world <= cfg.kv_heads:
        if cfg.kv_heads % world:
            raise ValueError(f"{cfg.kv_heads} KV heads do not split over {world} ranks")
        per = cfg.kv_heads // world
        return rank * per * G, (rank + 1) * per * G, rank * per, (rank + 1) * per
    if world % cfg.kv_heads:
        raise ValueError(f"{world} ranks do not split {cfg.kv_heads} KV heads")
    share = world // cfg.kv_heads
    kv = rank // share
    j = rank % share
    q0 = kv * G + (G * j) // share
    q1 = kv * G + (G * (j + 1)) // share
    return q0, q1, kv, kv + 1


def vocab_split(cfg: Qwen2Config, rank: int, world: int):
    """This rank's lm_head rows [v0, v1) (multiples of 64 except the last end)."""
    vb = (cfg.vocab + 63) // 64
    v0 = (vb * rank // world) * 64
    v1 = min(cfg.vocab, (vb * (rank + 1) // world) * 64) if rank + 1 < world else cfg.vocab
    return v0, v1


def inter_split(cfg: Qwen2Config, rank: int, world: int):
    """This rank's intermediate columns, multiples of 64."""
    kb = cfg.intermediate // 64
    i0 = (kb * rank // world) * 64
    i1 = (kb * (rank + 1) // world) * 64 if rank + 1 < world else cfg.intermediate
    return i0, i1


# ------------------------------------------------------------------ a random-init model

@dataclass
class Checkpoint:
    """A model in the reference's compiled format: per layer and projection the compress.rs key set
    (on the GPU), per projection (t4, t8), dense f32 norms and biases, the f16 embedding table."""
    cfg: Qwen2Config
    blocks: List[Dict[str, dict]]            # [layer][proj] -> compress_tensor_to_saccade() dict
    thresholds: List[Dict[str, tuple]]       # [layer][proj] -> (t4, t8)
    norms: List[Dict[str, torch.Tensor]]     # [layer] -> {"input", "post"} f32 [hidden]
    biases: List[Dict[str, torch.Tensor]]    # [layer] -> {"q", "k", "v"} f32
    final_norm: torch.Tensor
    embed: torch.Tensor                      # f16 [vocab, hidden]
    lm_head: Optional[torch.Tensor] = None   # f16 [vocab, hidden] (None: tied)


def random_checkpoint(cfg: Qwen2Config, seed: int = 42, fill: float = 0.01, device="cuda:0",
                      layers: Optional[int] = None) -> Checkpoint:
    """Random init (linears N(0, 0.02), q/k/v biases N(0, 0.01), norms 1, embeddings N(0, 0.02)
    rounded to f16), each linear packed on the GPU with the percentile threshold at `fill`.  The
    router thresholds start at +inf (nothing routed); calibrate() sets them."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    nl = cfg.layers if layers is None else layers
    blocks, thr, norms, biases = [], [], [], []
    inf = float(np.finfo(np.float32).max)
    for _ in range(nl):
        lb = {}
        for name in PROJ:
            n, k = cfg.proj_shape(name)
            w = torch.randn(n, k, device=dev, generator=g) * 0.02
            t = compute_percentile_threshold(w, fill)
            lb[name] = compress_tensor_to_saccade(w, t)
            del w
        blocks.append(lb)
        thr.append({name: (inf, inf) for name in PROJ})
        norms.append({"input": torch.ones(cfg.hidden, device=dev), "post": torch.ones(cfg.hidden, device=dev)})
        biases.append({name: torch.randn(cfg.proj_shape(name)[0], device=dev, generator=g) * 0.01
                       for name in ("q", "k", "v")})
    embed = (torch.randn(cfg.vocab, cfg.hidden, device=dev, generator=g) * 0.02).to(torch.float16)
    lm = None if cfg.tie_embeddings else (torch.randn(cfg.vocab, cfg.hidden, device=dev, generator=g) * 0.02).to(
        torch.float16)
    return Checkpoint(cfg, blocks, thr, norms, biases, torch.ones(cfg.hidden, device=dev), embed, lm)


def _u32(t):
    return t.view(torch.int32) if t.dtype == torch.uint32 else t


# ------------------------------------------------------------------ the model

class Qwen2Model:
    """Qwen2Model::forward on one GPU, or one rank of a tensor-parallel group (tp = (rank, world,
    process_group) with NCCL).  Serves up to `max_batch` sequences of up to `max_pos` positions."""

    def __init__(self, ck: Checkpoint, device=None, max_batch: int = 1, max_pos: int = 512, mode: str = "fast",
                 tp=None, fused_route="none"):
        """fused_route: where a group of linears runs the 9..64-token launch, its router runs in the
        kernel that writes its input instead of a router launch of its own: "norm" for q,k,v and
        gate,up (the RMSNorm kernel), "all" also for down on one GPU (the SiLU * up kernel).  The
        results are the same bits either way; "none" (separate router launches) is the default
        because it measured fastest in the captured Qwen2-7B batch-64 decode step (13.68 ms against
        13.83 ms "norm" and 14.35 ms "all")."""
        self.cfg = cfg = ck.cfg
        if fused_route is True or fused_route is False:
            fused_route = "all" if fused_route else "none"
        if fused_route not in ("none", "norm", "all"):
            raise ValueError("fused_route is 'none', 'norm' or 'all'")
        self.fused_route = fused_route
        self.device = dev = torch.device(ck.embed.device if device is None else device)
        self.max_batch, self.max_pos = max_batch, max_pos
        self.rank, self.world, self.group = tp if tp is not None else (0, 1, None)
        self.q0, self.q1, self.k0, self.k1 = head_split(cfg, self.rank, self.world)
        self.i0, self.i1 = inter_split(cfg, self.rank, self.world)
        self.nh, self.nkv = self.q1 - self.q0, self.k1 - self.k0
        hd = cfg.head_dim
        self.layers = []
        for li, lb in enumerate(ck.blocks):
            th = ck.thresholds[li]
            L = {}
            for name in PROJ:
                n, k = cfg.proj_shape(name)
                b = lb[name]
                rng = {"q": (self.q0 * hd, self.q1 * hd), "k": (self.k0 * hd, self.k1 * hd),
                       "v": (self.k0 * hd, self.k1 * hd), "gate": (self.i0, self.i1), "up": (self.i0, self.i1),
                       "o": (self.q0 * hd, self.q1 * hd), "down": (self.i0, self.i1)}[name]
                kind = "rows" if name in ("o", "down") else "columns"
                shard = None if self.world == 1 else (kind + "_range", rng[0], rng[1])
                sp = None
                if "delta_row_ptrs" in b:
                    sp = SparseDeltaMatrix(b["delta_row_ptrs"], b["delta_col_indices"], b["delta_values"],
                                           b["delta_scale"])
                L[name] = SaccadeLinearOp(b["packed_base"], b["scale_base"], sp, SaccadeConfig(*th[name]), n, k,
                                          device=dev, mode=mode, shard=shard)
            L["qkv"] = SaccadeLinearGroup([L["q"], L["k"], L["v"]])
            L["gateup"] = SaccadeLinearGroup([L["gate"], L["up"]])
            if self.world == 1:
                L["downg"] = SaccadeLinearGroup([L["down"]])
            bq = ck.biases[li]
            L["bias"] = [bq["q"][self.q0 * hd:self.q1 * hd].to(dev, torch.float32).contiguous(),
                         bq["k"][self.k0 * hd:self.k1 * hd].to(dev, torch.float32).contiguous(),
                         bq["v"][self.k0 * hd:self.k1 * hd].to(dev, torch.float32).contiguous()]
            L["norm_in"] = ck.norms[li]["input"].to(dev, torch.float32).contiguous()
            L["norm_post"] = ck.norms[li]["post"].to(dev, torch.float32).contiguous()
            self.layers.append(L)
        self.final_norm = ck.final_norm.to(dev, torch.float32).contiguous()
        self.embed = ck.embed.to(dev).contiguous()
        self.v0, self.v1 = vocab_split(cfg, self.rank, self.world)
        table = (ck.embed if ck.lm_head is None else ck.lm_head).to(dev)
        if self.world > 1:
            table = table[self.v0:self.v1].contiguous()
        self.lm_head_t = table.t()  # [hidden, vocab slice] view, f16
        cos, sin = rope_tables(cfg, max_pos)
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        shape = (max_batch, self.nkv, max_pos, hd)
        self.k_cache = [torch.zeros(shape, dtype=torch.float32, device=dev) for _ in self.layers]
        self.v_cache = [torch.zeros(shape, dtype=torch.float32, device=dev) for _ in self.layers]
        self.status = torch.zeros(4, dtype=torch.int32, device=dev)
        self._bufs = {}
        torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
        torch.backends.cuda.matmul.allow_tf32 = False

    # -------------------------------------------------------------- buffers
    def _buf(self, key, shape, dtype):
        b = self._bufs.get(key)
        if b is None or b.shape != torch.Size(shape) or b.dtype != dtype:
            b = torch.empty(shape, dtype=dtype, device=self.device)
            self._bufs[key] = b
        return b

    def _routing(self, key, group: SaccadeLinearGroup, n_layers: int, T: int, fuse: bool):
        """The fused router's buffers for `group` at T tokens (shared by every layer: the stream
        orders their uses), or None where the group routes by itself."""
        k = ("route",) + key + (T,)
        if k not in self._bufs:
            self._bufs[k] = GroupRouting(n_layers, T, self.device) if fuse and group.takes_routing(T) else None
        return self._bufs[k]

    def _stream(self):
        return ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)

    def _all_reduce(self, t: torch.Tensor):
        if self.world > 1:
            torch.distributed.all_reduce(t, group=self.group)

    # -------------------------------------------------------------- one pass over the layers
    def forward_tokens(self, ids: torch.Tensor, slot: torch.Tensor, pos: torch.Tensor, last: torch.Tensor,
                       max_query_pos: int) -> torch.Tensor:
        """Runs T tokens (ids [T] int64, cache slot [T] and position [T] int32) through the model,
        appending their keys and values; returns the f32 logits [len(last), v1 - v0] of the tokens
        at indices `last` (int64) over this rank's vocabulary slice [v0, v1) (all of it on one GPU)."""
        cfg, dev = self.cfg, self.device
        T = ids.numel()
        H, hd = cfg.hidden, cfg.head_dim
        st = self._stream()
        resid = self._buf(("resid", T), (T, H), torch.float32)
        check(LIB.sc_qwen2_embed(ids.data_ptr(), T, self.embed.data_ptr(), cfg.vocab, H, resid.data_ptr(),
                                 self.status.data_ptr(), st))
        x16 = self._buf(("x16", T), (T, H), torch.float16)
        q = self._buf(("q", T), (T, self.nh * hd), torch.float32)
        k = self._buf(("k", T), (T, self.nkv * hd), torch.float32)
        v = self._buf(("v", T), (T, self.nkv * hd), torch.float32)
        a16 = self._buf(("a16", T), (T, self.nh * hd), torch.float16)
        delta = self._buf(("delta", T), (T, H), torch.float32)
        ni = self.i1 - self.i0
        g16 = self._buf(("g16", T), (T, ni), torch.float16)
        u16 = self._buf(("u16", T), (T, ni), torch.float16)
        m16 = self._buf(("m16", T), (T, ni), torch.float16)
        scratch_bytes = int(LIB.sc_qwen2_attention_scratch(T, self.nh, self.nkv, hd, self.max_pos))
        scratch = self._buf(("attn", T), (max(1, scratch_bytes // 4),), torch.float32)
        have_delta = False
        L0 = self.layers[0]
        fuse_norm = self.fused_route in ("norm", "all")
        r_qkv = self._routing(("qkv",), L0["qkv"], 3, T, fuse_norm)
        r_gu = self._routing(("gateup",), L0["gateup"], 2, T, fuse_norm)
        r_down = (self._routing(("down",), L0["downg"], 1, T, self.fused_route == "all")
                  if self.world == 1 else None)
        eps = ctypes.c_float(cfg.eps)
        for li, L in enumerate(self.layers):
            dptr = delta.data_ptr() if have_delta else None
            if r_qkv is not None:
                check(LIB.sc_qwen2_add_rmsnorm_route(resid.data_ptr(), dptr, L["norm_in"].data_ptr(), T, H, eps,
                                                     x16.data_ptr(), L["qkv"]._h, r_qkv.mask_p, r_qkv.ridx_p,
                                                     r_qkv.count_p, r_qkv.counter.data_ptr(), st))
                L["qkv"].forward_routed(x16, r_qkv, out_dtype=torch.float32, outs=[q, k, v], biases=L["bias"])
            else:
                check(LIB.sc_qwen2_add_rmsnorm(resid.data_ptr(), dptr, L["norm_in"].data_ptr(), T, H, eps,
                                               x16.data_ptr(), _lib.SC_F16, st))
                L["qkv"].forward(x16, out_dtype=torch.float32, outs=[q, k, v], biases=L["bias"])
            check(LIB.sc_qwen2_rope_append(q.data_ptr(), k.data_ptr(), v.data_ptr(), self.cos.data_ptr(),
                                           self.sin.data_ptr(), slot.data_ptr(), pos.data_ptr(), T, self.nh, self.nkv,
                                           hd, self.max_pos, self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(),
                                           st))
            check(LIB.sc_qwen2_attention(q.data_ptr(), self.k_cache[li].data_ptr(), self.v_cache[li].data_ptr(),
                                         slot.data_ptr(), pos.data_ptr(), T, self.nh, self.nkv, hd, self.max_pos,
                                         max_query_pos, scratch.data_ptr(), scratch.numel() * 4, a16.data_ptr(), st))
            self._row_layer(L["o"], a16, delta, ("o", T))
            if r_gu is not None:
                check(LIB.sc_qwen2_add_rmsnorm_route(resid.data_ptr(), delta.data_ptr(), L["norm_post"].data_ptr(), T,
                                                     H, eps, x16.data_ptr(), L["gateup"]._h, r_gu.mask_p, r_gu.ridx_p,
                                                     r_gu.count_p, r_gu.counter.data_ptr(), st))
                L["gateup"].forward_routed(x16, r_gu, outs=[g16, u16])
            else:
                check(LIB.sc_qwen2_add_rmsnorm(resid.data_ptr(), delta.data_ptr(), L["norm_post"].data_ptr(), T, H,
                                               eps, x16.data_ptr(), _lib.SC_F16, st))
                L["gateup"].forward(x16, outs=[g16, u16])
            if r_down is not None:
                check(LIB.sc_qwen2_silu_mul_route(g16.data_ptr(), u16.data_ptr(), T, ni, m16.data_ptr(), L["downg"]._h,
                                                  r_down.mask_p, r_down.ridx_p, r_down.count_p,
                                                  r_down.counter.data_ptr(), st))
                L["downg"].forward_routed(m16, r_down, out_dtype=torch.float32, outs=[delta])
            else:
                check(LIB.sc_qwen2_silu_mul(g16.data_ptr(), u16.data_ptr(), T * ni, m16.data_ptr(), st))
                self._row_layer(L["down"], m16, delta, ("down", T))
            have_delta = True
        nl = last.numel()
        rl = self._buf(("rlast", nl), (nl, H), torch.float32)
        dl = self._buf(("dlast", nl), (nl, H), torch.float32)
        torch.index_select(resid, 0, last, out=rl)
        torch.index_select(delta, 0, last, out=dl)
        xn = self._buf(("xn", nl), (nl, H), torch.float32)
        check(LIB.sc_qwen2_add_rmsnorm(rl.data_ptr(), dl.data_ptr(), self.final_norm.data_ptr(), nl, H,
                                       ctypes.c_float(cfg.eps), xn.data_ptr(), _lib.SC_F32, st))
        return self._lm_head(xn)

    def _row_layer(self, op: SaccadeLinearOp, x16: torch.Tensor, out_f32: torch.Tensor, key):
        """o / down: y = f32(f16(acc)) (model.rs:61) into out_f32; on several ranks the rank's f32 partial
        sums and router sums are all-reduced, then routed and rounded."""
        if self.world == 1:
            op.forward(x16, out_dtype=torch.float32, out=out_f32)
            return
        T = x16.shape[0]
        part = self._buf(key + ("part",), (op.exchange_size(T),), torch.float32)
        op.forward_split(x16, part)
        self._all_reduce(part)
        op.finalize_split(part, T, self.world, out=out_f32)

    def _lm_head(self, xn: torch.Tensor) -> torch.Tensor:
        """logits = x . W^T with f16 W: x = hi + lo (f16 each), two f16 GEMMs with f32 accumulation."""
        nl = xn.shape[0]
        hilo = self._buf(("hilo", nl), (2 * nl, xn.shape[1]), torch.float16)
        hi = xn.to(torch.float16)
        hilo[:nl].copy_(hi)
        hilo[nl:].copy_((xn - hi.float()).to(torch.float16))
        p = torch.mm(hilo, self.lm_head_t, out_dtype=torch.float32)
        return p[:nl] + p[nl:]

    def undecided_routes(self) -> int:
        """Row-layer tokens routed on the f64 score inside the f32 error bound (tensor parallel only)."""
        if self.world == 1:
            return 0
        return int(sum(int(L[n].undecided.item()) for L in self.layers for n in ("o", "down")))

    def check_device(self):
        for L in self.layers:
            for name in PROJ:
                L[name].check_device()
        if int(self.status[0].item()) != 0:
            raise _lib.CTarqError(_lib.SC_EDEVICE, "a token id outside the vocabulary")


# ------------------------------------------------------------------ calibration and generation

def calibrate(ck: Checkpoint, prompt: torch.Tensor, pct=(0.75, 0.95), device=None, mode="fast",
              max_pos: Optional[int] = None) -> None:
    """ProfileRunner::calibrate per projection (calibration.rs:10-47) on the inputs each projection
    sees while `prompt` [B, S] runs through the model with nothing routed; writes ck.thresholds.
    The model runs on `device` (default: the checkpoint's)."""
    B, S = prompt.shape
    device = ck.embed.device if device is None else device
    # unfused routers: the hooks below read each projection's input where its forward receives it
    model = Qwen2Model(ck, device, max_batch=B, max_pos=max_pos or S, mode=mode, fused_route="none")
    acts = {}
    orig = {}
    for li, L in enumerate(model.layers):
        for name in ("q", "o", "gate", "down"):
            op = L[name]
            orig[(li, name)] = op.forward

            def hook(x, *a, _li=li, _name=name, _f=op.forward, **kw):
                acts[(_li, _name)] = x.detach().clone()
                return _f(x, *a, **kw)
            op.forward = hook
        for gname, first in (("qkv", "q"), ("gateup", "gate")):
            grp = L[gname]

            def ghook(x, *a, _li=li, _first=first, _f=grp.forward, **kw):
                acts[(_li, _first)] = x.detach().clone()
                return _f(x, *a, **kw)
            grp.forward = ghook
    ids, slot, pos = prefill_indices(prompt.to(model.device))
    model.forward_tokens(ids, slot, pos, torch.tensor([ids.numel() - 1], device=model.device), S - 1)
    torch.cuda.synchronize(model.device)
    for li in range(len(ck.blocks)):
        for name, src in (("q", "q"), ("k", "q"), ("v", "q"), ("o", "o"), ("gate", "gate"), ("up", "gate"),
                          ("down", "down")):
            ck.thresholds[li][name] = ProfileRunner.calibrate(acts[(li, src)], *pct)
    del model


def prefill_indices(prompt: torch.Tensor):
    """ids, cache slots and positions of a [B, S] prompt, flattened batch-major."""
    B, S = prompt.shape
    dev = prompt.device
    ids = prompt.reshape(-1).to(torch.int64).contiguous()
    slot = torch.arange(B, device=dev, dtype=torch.int32).repeat_interleave(S)
    pos = torch.arange(S, device=dev, dtype=torch.int32).repeat(B)
    return ids, slot, pos


class GreedyDecoder:
    """Prefill, then greedy decoding one token per sequence per step (verify.rs:98-130), each decode
    step replayed as one CUDA graph: token ids in, argmax token ids out (the step also copies them
    to its own input, so back-to-back replays decode autonomously)."""

    def __init__(self, model: Qwen2Model, batch: int):
        self.model = model
        self.B = batch
        dev = model.device
        self.ids = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.slot = torch.arange(batch, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.last = torch.arange(batch, dtype=torch.int64, device=dev)
        self.next = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.logits = None
        self.graph = None
        self.stream = torch.cuda.Stream(device=dev)
        self._xchg = {}  # rows -> ((rows, 2), (world, rows, 2)) f32 buffers of the tensor-parallel argmax

    def argmax(self, logits: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Greedy token of each row: over this rank's vocabulary slice, then (tensor parallel) the
        first of the ranks' maxima, so ties go to the smallest id as with one argmax."""
        m = self.model
        if m.world == 1:
            return torch.argmax(logits, dim=-1, out=out)
        n = logits.shape[0]
        if n not in self._xchg:
            self._xchg[n] = (torch.zeros(n, 2, dtype=torch.float32, device=m.device),
                             torch.zeros(m.world, n, 2, dtype=torch.float32, device=m.device))
        cand, gath = self._xchg[n]
        val, idx = torch.max(logits, dim=-1)
        cand[:, 0].copy_(val)
        cand[:, 1].copy_(idx + m.v0)  # ids < 2^24 are exact in f32
        torch.distributed.all_gather_into_tensor(gath, cand, group=m.group)
        best = torch.argmax(gath[:, :, 0], dim=0)  # first rank holding the maximum
        out.copy_(gath[:, :, 1].gather(0, best[None, :])[0].to(torch.int64))
        return out

    def prefill(self, prompt: torch.Tensor, chunk: int = 0) -> torch.Tensor:
        """Runs the prompts [B, S] (`chunk` sequences per pass, all at once by default) and returns the
        greedy first tokens [B]."""
        m = self.model
        B, S = prompt.shape
        chunk = chunk or B
        first = torch.empty(B, dtype=torch.int64, device=m.device)
        self.prefill_logits = []
        for b0 in range(0, B, chunk):
            b1 = min(B, b0 + chunk)
            ids, slot, pos = prefill_indices(prompt[b0:b1].to(m.device))
            slot += b0
            last = torch.arange(b1 - b0, device=m.device, dtype=torch.int64) * S + (S - 1)
            logits = m.forward_tokens(ids, slot, pos, last, S - 1)
            self.argmax(logits, first[b0:b1])
            self.prefill_logits.append(logits)
        self.pos.fill_(S)
        self.next.copy_(first)
        self.ids.copy_(first)
        return first

    def _step(self):
        self.logits = self.model.forward_tokens(self.ids, self.slot, self.pos, self.last, self.model.max_pos - 1)
        self.argmax(self.logits, self.next)
        self.ids.copy_(self.next)
        self.pos.add_(1)

    def capture(self):
        """Records one decode step as a CUDA graph, after the prefill (whose larger calls size the
        workspaces first), following one eager step that sizes the step's buffers (its cache writes
        are rewritten by the first replay at the same position)."""
        self.stream.wait_stream(torch.cuda.current_stream(self.model.device))
        ids0 = self.ids.clone()
        with torch.cuda.stream(self.stream):
            self._step()
            self.pos.sub_(1)
            self.ids.copy_(ids0)
        self.stream.synchronize()
        self.launches_per_step = int(LIB.sc_launch_count())
        self.graph = torch.cuda.CUDAGraph()
        with no_gc(), torch.cuda.graph(self.graph, stream=self.stream):
            self._step()
        self.launches_per_step = int(LIB.sc_launch_count()) - self.launches_per_step
        self.stream.synchronize()
        flush_deferred()

    def step(self, ids: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step on the decoder's stream: ids [B] (device or pinned host; default: the
        previous step's argmax, already in place) -> argmax ids [B] (device)."""
        with torch.cuda.stream(self.stream):
            if ids is not None:
                self.ids.copy_(ids, non_blocking=True)
            if self.graph is not None:
                self.graph.replay()
            else:
                self._step()
        return self.next

    def generate(self, prompt: torch.Tensor, steps: int, record_logits: bool = False, chunk: int = 0,
                 graph: bool = True):
        """Greedy tokens [B, steps] (and the top-2 logit gap of each step when record_logits; one GPU),
        each decode step a replay of the captured graph unless graph=False."""
        self.stream.wait_stream(torch.cuda.current_stream(self.model.device))
        with torch.cuda.stream(self.stream):
            tok = self.prefill(prompt, chunk)
            out, gaps = [tok.clone()], []
            if record_logits:
                first = torch.cat(self.prefill_logits)
                top = torch.topk(first, 2, dim=-1).values
                gaps.append((top[:, 0] - top[:, 1]).cpu())
        if graph and self.graph is None:
            self.capture()
        for _ in range(steps - 1):
            nxt = self.step()
            self.stream.synchronize()
            out.append(nxt.clone())
            if record_logits:
                top = torch.topk(self.logits, 2, dim=-1).values
                gaps.append((top[:, 0] - top[:, 1]).cpu())
        toks = torch.stack(out, dim=1)
        return (toks, torch.stack(gaps, dim=1)) if record_logits else toks
