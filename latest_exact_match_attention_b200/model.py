"""The LEMA transformer, inference only, on the B200 kernels.

Same architecture and parameter names as code/lema/model.py (pre-RMSNorm, SwiGLU MLP,
untied head, no biases, no positional scheme), so a state dict trained by the reference
loads unchanged. Only the exact ("hard") LEMA op is served: attention kinds other than
"lema" and the training-time surrogate are outside this package.

Where the time goes, and what replaced it:

    Block.gpu_pre    norm1 -> K1 (lema_proj_codes: q/k GEMM + sign pack on the tensor
                     cores, z never stored) + v_proj          code/lema/model.py:224-227
    Attention        the exact op: K2 (lema_prefill_match: latest match + gather)
                                                               code/lema/model.py:199-202
    Block.forward    with a store: codes -> K3 (lema_store_exchange, the store in HBM)
                                                               code/lema/model.py:249-253
    Transformer.forward(idx, cache=)                           code/lema/model.py:337-363

K1 serves d_qk = 32 with bf16 weights and dim % 64 == 0 (every benchmark configuration);
other shapes project with torch and pack with lema_pack_codes.
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib
from ._lib import DTYPE_TAG, call, check_status, device_status, ptr, stream_handle
from .attention import pack_codes, prefill_match, proj_codes

ATTN_KINDS = ("lema",)


def _pad128(n) -> int:
    return -(-int(n) // 128) * 128


@dataclass
class ModelConfig:
    """Fields and defaults of code/lema/model.py:35-87 (`ModelConfig`): d_qk and d_v default
    to dim // num_heads, dim_ff to 8 * dim / 3, and vocab_size and dim_ff are rounded up to a
    multiple of 128."""
    vocab_size: int
    depth: int
    dim: int
    num_heads: int
    d_qk: int = 0
    d_v: int = 0
    dim_ff: int = 0
    num_kv_heads: int = 0
    attn: str = "lema"
    pos: str = "nope"
    rope_base: float = 10000.0
    gdn_expand_v: int = 2
    norm_eps: float = 1e-5

    def __post_init__(self):
        if self.attn not in ATTN_KINDS:
            raise ValueError(f"this build serves attn='lema' only (the exact op); got "
                             f"{self.attn!r}")
        if self.pos != "nope":
            raise ValueError(f"a LEMA model has no positional scheme; pos={self.pos!r}")
        if (not self.d_qk or not self.d_v) and self.dim % self.num_heads:
            raise ValueError(f"dim {self.dim} is not divisible by num_heads {self.num_heads}")
        head = self.dim // self.num_heads
        self.d_qk = self.d_qk or head
        self.d_v = self.d_v or head
        self.dim_ff = _pad128(self.dim_ff or 8 * self.dim / 3)
        self.vocab_size = _pad128(self.vocab_size)
        self.num_kv_heads = self.num_kv_heads or self.num_heads
        if self.num_kv_heads != self.num_heads:
            raise ValueError("grouped-query attention is not defined for LEMA "
                             "(num_kv_heads must equal num_heads)")
        if self.d_qk > 64:
            raise ValueError(f"d_qk {self.d_qk} > 64: codes must pack into one uint64")

    @classmethod
    def from_dict(cls, d: dict) -> "ModelConfig":
        """A config from a saved dict (a checkpoint's config.json); keys that are not
        fields of this config are ignored."""
        known = {f.name: d[f.name] for f in dataclasses.fields(cls) if f.name in d}
        return cls(**known)

    def summary(self) -> str:
        return (f"{self.depth}L d{self.dim} h{self.num_heads} d_qk {self.d_qk} d_v {self.d_v} "
                f"dim_ff {self.dim_ff} attn {self.attn}")


def rms_norm(norm: nn.RMSNorm, x: torch.Tensor) -> torch.Tensor:
    """`norm(x)` (code/lema/model.py:215-217, 264): one pass of lema_rms_norm for 16-bit rows
    on the GPU (torch's kernel reads the rows at under half the HBM rate at config 3), the
    module itself otherwise (fp32, CPU, odd widths)."""
    D = x.shape[-1]
    w = norm.weight
    if (x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and w is not None
            and w.dtype == x.dtype and D % 8 == 0 and x.is_contiguous()
            and x.data_ptr() % 16 == 0 and w.data_ptr() % 16 == 0):
        out = torch.empty_like(x)
        eps = norm.eps if norm.eps is not None else torch.finfo(x.dtype).eps
        call("lema_rms_norm", ptr(x), ptr(w), DTYPE_TAG[x.dtype], x.numel() // D, D, eps, ptr(out),
             stream_handle(x.device))
        return out
    return norm(x)


class SwiGLU(nn.Module):
    """down(silu(gate(x)) * up(x)), parameters named as code/lema/model.py:85-93. On a GPU, for
    bf16 prefill-sized inputs (at least FUSED_MIN_ROWS rows) the gate and up projections and
    the activation are one tcgen05 GEMM with SwiGLU in its epilogue (lema_gemm_swiglu, on the
    gate/up weights interleaved in blocks of 128 rows); otherwise one GEMM on the stacked
    weights and one activation kernel (lema_swiglu). `forward(x, residual)` adds the residual
    inside the down GEMM."""

    FUSED_MIN_ROWS = 4096  # below this the fused GEMM has too few 128-row tiles per SM

    def __init__(self, dim: int, dim_ff: int):
        super().__init__()
        self.gate = nn.Linear(dim, dim_ff, bias=False)
        self.up = nn.Linear(dim, dim_ff, bias=False)
        self.down = nn.Linear(dim_ff, dim, bias=False)
        self._wgu = None
        self._wil = None

    def gate_up_weight(self) -> torch.Tensor:
        g, u = self.gate.weight, self.up.weight
        key = (g.data_ptr(), u.data_ptr(), g._version, u._version)
        if self._wgu is None or self._wgu[0] != key:
            self._wgu = (key, torch.cat([g.detach(), u.detach()], 0).contiguous())
        return self._wgu[1]

    def gate_up_interleaved(self) -> torch.Tensor:
        """[2F, dim]: gate rows 128 b ... 128 b + 127, then the up rows of the same features."""
        g, u = self.gate.weight, self.up.weight
        key = (g.data_ptr(), u.data_ptr(), g._version, u._version)
        if getattr(self, "_wil", None) is None or self._wil[0] != key:
            Fd, dim = g.shape
            w = torch.stack([g.detach().view(Fd // 128, 128, dim), u.detach().view(Fd // 128, 128, dim)], 1)
            self._wil = (key, w.reshape(2 * Fd, dim).contiguous())
        return self._wil[1]

    def _fused_ok(self, x2) -> bool:
        Fd, dim = self.gate.weight.shape
        return (x2.dtype == torch.bfloat16 and x2.shape[0] >= self.FUSED_MIN_ROWS and Fd % 128 == 0
                and dim % 64 == 0 and x2.is_contiguous() and x2.data_ptr() % 16 == 0
                and self.gate.weight.dtype == torch.bfloat16 and torch.cuda.get_device_capability(x2.device)[0] == 10)

    def forward(self, x, residual=None):
        if not x.is_cuda or x.dtype not in DTYPE_TAG:
            y = self.down(F.silu(self.gate(x)) * self.up(x))
            return y if residual is None else residual + y
        lead, dim = x.shape[:-1], x.shape[-1]
        x2 = x.reshape(-1, dim)
        Fd = self.gate.weight.shape[0]
        act = torch.empty((x2.shape[0], Fd), dtype=x.dtype, device=x.device)
        if self._fused_ok(x2):
            call("lema_gemm_swiglu", ptr(x2), ptr(self.gate_up_interleaved()), x2.shape[0], dim, Fd,
                 ptr(act), ptr(device_status(x.device)), stream_handle(x.device))
        else:
            gu = x2 @ self.gate_up_weight().t()
            call("lema_swiglu", ptr(gu), DTYPE_TAG[x.dtype], x2.shape[0], Fd, ptr(act),
                 stream_handle(x.device))
        w = self.down.weight.t()
        y = act @ w if residual is None else torch.addmm(residual.reshape(-1, dim), act, w)
        return y.view(*lead, dim)


class Attention(nn.Module):
    """A LEMA head group: projections named as code/lema/model.py:160-163; the op is always
    the exact one (`hard`), computed from codes."""

    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        self.kind = "lema"
        H = cfg.num_heads
        self.q_proj = nn.Linear(cfg.dim, H * cfg.d_qk, bias=False)
        self.k_proj = nn.Linear(cfg.dim, H * cfg.d_qk, bias=False)
        self.v_proj = nn.Linear(cfg.dim, H * cfg.d_v, bias=False)
        self.o_proj = nn.Linear(H * cfg.d_v, cfg.dim, bias=False)
        self.hard = True
        self._wqk = None        # (key, stacked [q_proj; k_proj] weight) for K1

    def project(self, x):
        """[B, T, dim] -> query and key pre-activations and values, [B, H, T, d]."""
        B, T, _ = x.shape
        c = self.cfg
        zq = self.q_proj(x).view(B, T, c.num_heads, c.d_qk).transpose(1, 2)
        zk = self.k_proj(x).view(B, T, c.num_heads, c.d_qk).transpose(1, 2)
        v = self.v_proj(x).view(B, T, c.num_heads, c.d_v).transpose(1, 2)
        return zq, zk, v

    def merge(self, y):
        B, _, T, _ = y.shape
        return self.o_proj(y.transpose(1, 2).reshape(B, T, -1))

    def _k1_ok(self, x) -> bool:
        w = self.q_proj.weight
        return (self.cfg.d_qk == 32 and x.is_cuda and x.dtype == torch.bfloat16
                and w.dtype == torch.bfloat16 and self.cfg.dim % 64 == 0)

    def stacked_qk(self) -> torch.Tensor:
        """[q_proj.weight; k_proj.weight], rebuilt only when either weight changes."""
        q, k = self.q_proj.weight, self.k_proj.weight
        key = (q.data_ptr(), k.data_ptr(), q._version, k._version)
        if self._wqk is None or self._wqk[0] != key:
            self._wqk = (key, torch.cat([q.detach(), k.detach()], 0).contiguous())
        return self._wqk[1]

    def exact(self, qc, kc, v):
        """The exact op on codes and values: [B, H, T, d_v] retrieved rows (zeros on a miss),
        as a transposed view of [B, T, H, d_v] memory -- what `merge` reads without a copy.
        v may be any [B, H, T, d_v] view with unit last stride (the projection's transposed
        output): the gather reads it in place."""
        B, H, T = qc.shape
        dv = v.shape[-1]
        if v.stride(-1) != 1:
            v = v.contiguous()
        es = v.element_size()
        out = torch.empty((B, T, H, dv), dtype=v.dtype, device=v.device)
        q2, k2 = qc.reshape(B * H, T).contiguous(), kc.reshape(B * H, T).contiguous()
        cb = 4 if q2.dtype == torch.int32 else 8
        nb = int(_lib.lib().lema_prefill_workspace_bytes(B * H, T, cb))
        ws = torch.empty(nb, dtype=torch.uint8, device=v.device) if nb else None
        call("lema_prefill_match_strided", ptr(q2), ptr(k2), cb, B * H, T, None, ptr(v), dv * es,
             ptr(out), H, v.stride(0) * es, v.stride(1) * es, v.stride(2) * es,
             T * H * dv * es, dv * es, H * dv * es, ptr(ws), nb, ptr(device_status(v.device)),
             stream_handle(v.device))
        return out.transpose(1, 2)

    def codes(self, x):
        """[B, T, dim] (normalised) -> (qcodes [B, H, T], kcodes [B, H, T], v [B, H, T, d_v]).
        Codes are int32 (uint32 bit patterns) for d_qk <= 32, else int64."""
        B, T, _ = x.shape
        c = self.cfg
        if self._k1_ok(x):
            qc, kc = proj_codes(x, self.stacked_qk(), c.num_heads, c.num_heads)
            v = self.v_proj(x).view(B, T, c.num_heads, c.d_v).transpose(1, 2)
            return qc, kc, v
        zq, zk, v = self.project(x)
        return pack_codes(zq, narrow=True), pack_codes(zk, narrow=True), v

    def forward(self, x):
        """The exact op over the whole sequence (no store): code/lema/attention.py:135-158."""
        qc, kc, v = self.codes(x)
        B, H, T = qc.shape
        vv = v.reshape(B * H, T, -1) if v.is_contiguous() else v.contiguous().view(B * H, T, -1)
        _, y = prefill_match(qc.reshape(B * H, T), kc.reshape(B * H, T), vv, want_src=False)
        return self.merge(y.view(B, H, T, -1))


class Block(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.norm1 = nn.RMSNorm(cfg.dim, eps=cfg.norm_eps)
        self.attn = Attention(cfg)
        self.norm2 = nn.RMSNorm(cfg.dim, eps=cfg.norm_eps)
        self.mlp = SwiGLU(cfg.dim, cfg.dim_ff)
        self.seg = None

    def gpu_pre(self, x):
        """Normalise, project and pack: the codes the store needs and the values
        (code/lema/model.py:224-227)."""
        return self.attn.codes(rms_norm(self.norm1, x))

    def gpu_post(self, x, got):
        """Merge the retrieved values and finish the layer: x + o_proj(merged heads) as one
        GEMM with the residual added in, then x + mlp(norm2(x)) likewise."""
        B, H, T, dv = got.shape
        dim = x.shape[-1]
        y = got.transpose(1, 2).reshape(B * T, H * dv)
        x = torch.addmm(x.reshape(B * T, dim), y, self.attn.o_proj.weight.t()).view(B, T, dim)
        return self.mlp(rms_norm(self.norm2, x), residual=x)

    def forward(self, x, store=None):
        if store is not None:
            pre, post = self.seg or (self.gpu_pre, self.gpu_post)
            qc, kc, v = pre(x)
            return post(x, store.exchange(qc, kc, v))
        qc, kc, v = self.gpu_pre(x)           # the same codes and values as the store path
        return self.gpu_post(x, self.attn.exact(qc, kc, v))


class Transformer(nn.Module):
    def __init__(self, cfg: ModelConfig):
        super().__init__()
        self.cfg = cfg
        self.tok_emb = nn.Embedding(cfg.vocab_size, cfg.dim)
        self.blocks = nn.ModuleList(Block(cfg) for _ in range(cfg.depth))
        self.norm_f = nn.RMSNorm(cfg.dim, eps=cfg.norm_eps)
        self.lm_head = nn.Linear(cfg.dim, cfg.vocab_size, bias=False)
        self._init_weights()

    def _init_weights(self):
        """The reference's random init (code/lema/model.py:269-281): N(0, 1/fan_in) for every
        Linear, N(0, 1/dim) for the embedding, and the two residual-branch outputs of each
        block (o_proj, mlp.down) scaled by 1/sqrt(2 * depth)."""
        for m in self.modules():
            if isinstance(m, nn.Linear):
                nn.init.normal_(m.weight, mean=0.0, std=1.0 / math.sqrt(m.weight.shape[1]))
            elif isinstance(m, nn.Embedding):
                nn.init.normal_(m.weight, mean=0.0, std=1.0 / math.sqrt(self.cfg.dim))
        for b in self.blocks:
            for lin in (b.attn.o_proj, b.mlp.down):
                lin.weight.data.mul_(1.0 / math.sqrt(2 * self.cfg.depth))

    def lema_layers(self):
        return [b.attn for b in self.blocks]

    def set_hard(self, hard: bool = True):
        if not hard:
            raise ValueError("this build serves the exact (hard) op only")

    def new_cache(self, place: str = "hbm", **kw):
        """The retrieval cache for this model, in device memory (the store is HBM-resident;
        place "ram" is accepted for the reference's call sites and means the same).
        Keywords as code/lema/cache.py:313-355: max_cache_len= or capacity=, max_load=,
        batch=, dtype= (default: the model's), codes_hook=."""
        from .cache import LemaCache
        if place not in ("hbm", "vram", "ram"):
            raise ValueError(f"place must be 'hbm' (or 'ram'/'vram', the same device store), "
                             f"got {place!r}")
        p = next(self.parameters())
        kw.setdefault("dtype", p.dtype)
        kw.setdefault("device", p.device)
        kw.pop("pin", None)
        return LemaCache(self.cfg, **kw)

    @torch.no_grad()
    def forward(self, idx, *, cache=None, return_logits=True):
        """forward(x): the whole batch, no state. forward(x, cache=c): queries also match
        every key already in `c`, and this call's keys are added to it (prefill in pieces,
        or one decode step); `return_logits=False` skips the head."""
        x = self.tok_emb(idx)
        for li, blk in enumerate(self.blocks):
            x = blk(x, store=(cache.layer(li) if cache is not None else None))
        if cache is not None:
            cache.t += idx.shape[-1]
        out = self.lm_head(rms_norm(self.norm_f, x)) if return_logits else None
        # device-side conditions of this forward's kernels (a bounded wait that ran out):
        # raised here, once per forward, outside graph capture
        check_status(x.device, "Transformer.forward")
        return out

    def n_params(self, embedding: bool = True) -> int:
        """Parameter count; embedding=False leaves out the token embedding and the head."""
        skip = set() if embedding else {id(self.tok_emb.weight), id(self.lm_head.weight)}
        return sum(p.numel() for p in self.parameters() if id(p) not in skip)
