"""Timed CPU baseline: the reference engine's unfused torch path on host cores.

TEST/BENCH INFRASTRUCTURE ONLY: ``bench.py`` times this as ``cpu_baseline``
and as the ``--impl reference`` arm; the product path never imports it.

It restates what the reference runs for one decode layer's projections:
  * QKV: three ``F.linear`` calls (engine/attention.py:119-121);
  * gate-up: ``F.silu(F.linear(x, Wg)) * F.linear(x, Wu)`` (engine/model.py:36-37);
  * MLA: reconstruct-K/V decode (engine/mla.py:206-262).
in the config's dtype (bf16) with every host thread torch will use.
"""

from __future__ import annotations

import os
import time

import torch
import torch.nn.functional as F

from .inputs import QWEN3_4B


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class DecodeProjections:
    """Weights of ``n_layers`` synthetic Qwen3-4B layers (bf16, N(0, 0.02))."""

    def __init__(self, n_layers: int = 2, M: int = 1, seed: int = 0, dtype=torch.bfloat16, n_random: int = 2):
        """Layers past the first ``n_random`` are clones of those (distinct
        memory, same values): the weight stream, not the values, sets the time,
        and drawing 4.7 GB of normals would take longer than timing them."""
        g = torch.Generator().manual_seed(seed)
        H, nq, nk, N = QWEN3_4B["hidden"], QWEN3_4B["n_q"], QWEN3_4B["n_k"], QWEN3_4B["inter"]
        self.layers = []
        for i in range(n_layers):
            if i < n_random:
                mk = lambda r: (torch.randn(r, H, generator=g) * 0.02).to(dtype)
                self.layers.append(dict(wq=mk(nq), wk=mk(nk), wv=mk(nk), wg=mk(N), wu=mk(N)))
            else:
                self.layers.append({k: v.clone() for k, v in self.layers[i % n_random].items()})
        self.x = torch.randn(M, H, generator=g).to(dtype)
        self.M = M

    @staticmethod
    def bytes_per_layer(M: int) -> int:
        H, nq, nk, N = QWEN3_4B["hidden"], QWEN3_4B["n_q"], QWEN3_4B["n_k"], QWEN3_4B["inter"]
        qkv = 2 * (nq + 2 * nk) * H + 2 * M * H + 2 * M * (nq + 2 * nk)
        gu = 2 * 2 * N * H + 2 * M * H + 2 * M * N
        return qkv + gu

    def run_layer(self, i: int):
        w = self.layers[i % len(self.layers)]
        x = self.x
        q, k, v = F.linear(x, w["wq"]), F.linear(x, w["wk"]), F.linear(x, w["wv"])
        y = F.silu(F.linear(x, w["wg"])) * F.linear(x, w["wu"])
        return q, k, v, y

    def run_step(self):
        """One decode pass: every layer's QKV and gate-up projections."""
        for i in range(len(self.layers)):
            self.run_layer(i)


def time_decode_projections(seconds: float = 10.0, M: int = 1, n_layers: int = 2, threads: int | None = None):
    """Run layer passes for about ``seconds``; returns a dict with GB/s."""
    threads = threads or host_cores()
    torch.set_num_threads(threads)
    dp = DecodeProjections(n_layers=n_layers, M=M)
    for i in range(2):
        dp.run_layer(i)
    n = 0
    t0 = time.perf_counter()
    while True:
        dp.run_layer(n)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    per_layer = el / n
    gbs = DecodeProjections.bytes_per_layer(M) / per_layer / 1e9
    return dict(gbs=gbs, layers=n, seconds=el, per_layer_s=per_layer, threads=threads)
