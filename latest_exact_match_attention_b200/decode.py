"""Single-token decoding as ONE CUDA graph per step.

The reference (code/lema/decode.py:183-240, `LemaDecoder`) replays depth + 1 graphs per
token with a host round trip between them: the store is a C++ table in host RAM, so every
layer copies its codes and values down, synchronises, exchanges on the CPU and copies the
retrieved rows back up. Here the store is in device memory and its exchange is a kernel
(K3), so the whole step -- embedding, every layer's codes, exchange and MLP, the head and
the choice of the next token -- is captured once and replayed as one graph. `step()` is
one replay: no host synchronisation, no copy across the bus. For small batches each layer's
store lookups stay on the step's path and its inserts run on a side branch of the graph beside
the layer's output projection and MLP (a decode step's items are distinct partitions, so the
split equals the combined exchange).

The captured work is exactly `Transformer.forward(tok, cache=...)`, the same segment
functions (`Block.gpu_pre`, `Block.gpu_post`) the eager path calls, so a replay reproduces
an eager step token for token.

Warm-up before the capture (the first calls allocate and set kernel attributes, which a
capture must not do) runs against a small scratch store, so the caller's store is left
exactly as it was; the capture itself launches nothing. A full store is reported through
the store's device status word: call `cache.check()` after stepping.
"""
from __future__ import annotations

import os

import torch

from .cache import HashStore, LemaCache
from .model import rms_norm


def _chooser(temperature: float):
    """Logits -> next token: argmax at temperature 0, else a sample from softmax(logits / T)
    by the Gumbel-max trick, argmax(logits / T + G) with G = -log(E), E ~ Exponential(1)
    (code/lema/decode.py:71-92 draws the same way), in fp32. Inside a graph the generator
    advances on every replay, so each step draws fresh noise."""
    if temperature <= 0:
        return lambda logits: logits.argmax(-1)

    def pick(logits):
        z = logits.float() / temperature
        g = torch.empty_like(z).exponential_().log_().neg_()
        return (z + g).argmax(-1)
    return pick


class LemaDecoder:
    """Greedy or sampled decoding of `cache.batch` streams, one graph replay per token.

    `tok` [B, 1] is the last token fed (e.g. the last prompt token after an eager prefill of
    the rest); after each `step()` it holds the newest generated token, on the device."""

    def __init__(self, model, cache: LemaCache, tok: torch.Tensor | None = None,
                 temperature: float = 0.0):
        cfg = model.cfg
        self.model, self.cache = model, cache
        B = cache.batch
        dev = next(model.parameters()).device
        self.tok = torch.zeros(B, 1, dtype=torch.long, device=dev)
        if tok is not None:
            self.tok.copy_(tok)
        choose = _chooser(temperature)
        views = [cache.layer(i) for i in range(cfg.depth)]
        side = torch.cuda.Stream(device=dev)
        self._staged = []
        # the split pays where the inserts are few (a small batch: measured at B = 1, worst-case
        # codes, load 0.95: 2.31 -> 2.10 ms per token); at B = 256 the side branch's 16384 items
        # per layer compete with the layer's GEMMs for SMs (1.66-1.76 ms combined, 1.80 split).
        # LEMA_DECODE_SPLIT=0/1 forces either (the same tokens).
        env = os.environ.get("LEMA_DECODE_SPLIT", "")[:1]
        split = env == "1" or (env != "0" and B * cfg.num_heads <= 4096)

        def step_fn():
            # each layer's lookups stay on the step's path; its inserts (needed only by the
            # next step's lookups) run on a side branch beside the layer's output projection
            # and MLP, joined at the end of the step. The staged buffers are kept referenced
            # so that nothing later in the capture reuses memory the side branch still reads.
            staged = []
            x = model.tok_emb(self.tok)
            cur = torch.cuda.current_stream(dev)
            for blk, view in zip(model.blocks, views):
                qc, kc, v = blk.gpu_pre(x)
                if split:
                    st, got = view.lookup(qc, kc, v)
                    side.wait_stream(cur)
                    with torch.cuda.stream(side):
                        view.insert(st)
                    staged.append(st)
                else:
                    got = view.exchange(qc, kc, v, check=False)
                x = blk.gpu_post(x, got)
            logits = model.lm_head(rms_norm(model.norm_f, x))
            self.tok.copy_(choose(logits).view(B, 1))
            if split:
                cur.wait_stream(side)
            self._staged = staged
            return logits

        # warm up on a scratch store (same row size and groups, room for the warm-up's keys)
        real = cache.store
        scratch = HashStore(cfg.d_v, groups=real.groups, dtype=real.dtype,
                            capacity=4 * cfg.depth * B * cfg.num_heads + 64, device=dev,
                            segments=cfg.depth)
        tok0 = self.tok.clone()
        cb = 4 if cfg.d_qk <= 32 else 8          # the codes' width (int32 or int64)
        real.reserve(B * cfg.num_heads, 1, cb)
        scratch.reserve(B * cfg.num_heads, 1, cb)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        try:
            for v in views:
                v.store = scratch
            with torch.no_grad(), torch.cuda.stream(s):
                for _ in range(2):
                    step_fn()
        finally:
            for v in views:
                v.store = real
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        del scratch
        self.graph = torch.cuda.CUDAGraph()
        with torch.no_grad(), torch.cuda.graph(self.graph):
            self.logits = step_fn()
        self.tok.copy_(tok0)

    def step(self) -> torch.Tensor:
        """One token for every stream; returns `tok` (device, [B, 1]), stream-ordered."""
        self.graph.replay()
        self.cache.t += 1
        return self.tok


def decoder(model, cache, tok=None, temperature: float = 0.0):
    """The decoder for a LEMA cache (code/lema/decode.py:243-248)."""
    return LemaDecoder(model, cache, tok, temperature)
