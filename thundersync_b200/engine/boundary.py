"""Graph cuts with owned fp32 adjoint ledgers (C17).

A :class:`Boundary` cuts the autograd graph at a shared node: consumers
attend to ``proxy`` tensors (detached twins of the node's outputs that share
storage and are gradient-requiring leaves). Every gradient a consumer's
backward deposits on a proxy is moved into an fp32 (fp64 for fp64 tensors)
ledger by a post-accumulate hook, so the node's own subgraph is backwarded
once with the summed adjoint instead of once per consumer (reference:
src/thundersync/engine/streaming.py:2647-2933).

Ledger arithmetic: the first contribution becomes the ledger by one widening
copy, later ones are added with a mixed-dtype ``add_`` that widens each
element exactly before the fp32 add, so the ledger holds the same bits as
"widen everything, then add in arrival order".
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable

import torch

__all__ = ["Boundary", "ledger_accumulate"]


def ledger_accumulate(ledgers: list[torch.Tensor | None], index: int, contribution: torch.Tensor) -> None:
    acc = ledgers[index]
    if acc is None:
        dtype = torch.float64 if contribution.dtype == torch.float64 else torch.float32
        ledgers[index] = contribution.to(dtype=dtype, copy=True)
    else:
        acc.add_(contribution)


@dataclass
class Boundary:
    real: list[torch.Tensor]
    proxy: list[torch.Tensor]
    capture_source: Callable[[], Any] | None = field(default=None, repr=False)
    _ledgers: list[torch.Tensor | None] = field(init=False, repr=False)
    _counts: list[int] = field(init=False, repr=False)
    _hooks: list[Any] = field(init=False, repr=False)
    _consumed: bool = field(default=False, init=False)
    lifetime_contributions: int = field(default=0, init=False)
    drains: int = field(default=0, init=False)
    _sources: set = field(default_factory=set, init=False, repr=False)
    # "torch": each contribution is added to its ledger when it arrives. "native" / "triton": contributions
    # wait (at most max_degree per tensor) and are reduced into the ledger in arrival order by one
    # fixed-order kernel launch (engine/boundary_adjoint.py) when max_degree are waiting or the ledger is read.
    reduce_backend: str = "torch"
    max_degree: int = 16
    _pending: list[list[torch.Tensor]] = field(init=False, repr=False)

    def __post_init__(self) -> None:
        if len(self.real) != len(self.proxy):
            raise ValueError("boundary real and proxy tensors must align")
        if not 1 <= self.max_degree <= 16:
            raise ValueError("max_degree must be in [1, 16]")
        self._ledgers = [None] * len(self.proxy)
        self._pending = [[] for _ in self.proxy]
        self._counts = [0] * len(self.proxy)
        self._hooks = []
        for i, p in enumerate(self.proxy):
            if not p.is_leaf or not p.requires_grad:
                raise ValueError("boundary proxies must be gradient-requiring leaves")
            self._hooks.append(p.register_post_accumulate_grad_hook(self._make_hook(i)))

    @classmethod
    def cut(cls, real: list[torch.Tensor], **kw) -> "Boundary":
        proxies = [r.detach().requires_grad_(True) for r in real]
        return cls(real=list(real), proxy=proxies, **kw)

    def _make_hook(self, index: int):
        def hook(p: torch.Tensor) -> None:
            g = p.grad
            p.grad = None
            if g is None:
                return
            self._add(index, g)
            self._counts[index] += 1
            self.lifetime_contributions += 1
            if self.capture_source is not None:
                src = self.capture_source()
                if src is not None:
                    self._sources.add(src)

        return hook

    # ------------------------------------------------------------ adjoints
    def _add(self, index: int, g: torch.Tensor) -> None:
        if self.reduce_backend == "torch":
            ledger_accumulate(self._ledgers, index, g)
            return
        self._pending[index].append(g.detach())
        if len(self._pending[index]) >= self.max_degree:
            self._flush(index)

    def _flush(self, index: int) -> None:
        """Reduce the waiting contributions of tensor ``index`` into its ledger, in arrival order."""
        pend = self._pending[index]
        if not pend:
            return
        self._pending[index] = []
        acc = self._ledgers[index]
        if acc is None:
            dtype = torch.float64 if pend[0].dtype == torch.float64 else torch.float32
            acc = torch.zeros(pend[0].shape, dtype=dtype, device=pend[0].device)
        if (acc.is_cuda and acc.dtype == torch.float32 and acc.is_contiguous()
                and pend[0].dtype in (torch.float32, torch.bfloat16)
                and all(t.is_cuda and t.dtype == pend[0].dtype for t in pend)):
            from thundersync_b200.ops._ext import native

            native().reduce_into(acc.view(-1), [t.contiguous().view(-1) for t in pend])
        else:
            for t in pend:
                acc.add_(t)
        self._ledgers[index] = acc

    def _flush_all(self) -> None:
        for i in range(len(self._pending)):
            self._flush(i)

    def accumulate_explicit(self, adjoints: list[torch.Tensor | None]) -> None:
        for i, a in enumerate(adjoints):
            if a is not None:
                self._add(i, a)
                self._counts[i] += 1
                self.lifetime_contributions += 1

    def has_adjoint(self) -> bool:
        return any(x is not None for x in self._ledgers) or any(self._pending)

    def peek(self) -> list[torch.Tensor | None]:
        self._flush_all()
        return list(self._ledgers)

    def drain(self) -> list[torch.Tensor | None]:
        """Take the ledgers (and reset them): one consumer's contribution."""
        self._flush_all()
        out = self._ledgers
        self._ledgers = [None] * len(self.proxy)
        self._counts = [0] * len(self.proxy)
        self.drains += 1
        return out

    def consume(self) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """(real, adjoint) pairs for the one backward of the node; marks consumed."""
        if self._consumed:
            raise RuntimeError("boundary adjoints were already consumed")
        self._consumed = True
        self._flush_all()
        pairs = []
        for r, a in zip(self.real, self._ledgers):
            if a is not None:
                pairs.append((r, a.to(r.dtype) if a.dtype != r.dtype else a))
        self._ledgers = [None] * len(self.proxy)
        return pairs

    @property
    def consumed(self) -> bool:
        return self._consumed

    def diagnostics(self) -> dict[str, Any]:
        return {
            "tensors": len(self.proxy),
            "contributions": list(self._counts),
            "lifetime_contributions": self.lifetime_contributions,
            "drains": self.drains,
            "sources": len(self._sources),
            "consumed": self._consumed,
        }

    def release(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []
        self.real = []
        self.proxy = []
        self._ledgers = []
        self._pending = []
