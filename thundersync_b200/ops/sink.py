"""Where native ops deposit parameter gradients.

A :class:`GradSink` redirects every parameter gradient an op's backward
produces into one flat fp32 buffer laid out by a :class:`ParamArena`, instead
of returning it to autograd's ``AccumulateGrad``. Linear weight gradients are
accumulated by the GEMM itself (``C += dYᵀ·X`` with fp32 ``C``), so a
per-trajectory gradient is never materialised in the parameter dtype and the
GRPO statistics can be the GEMM's accumulator directly.

The active sink is process-global, not thread-local: the autograd engine runs
CUDA backward functions on its own device thread. The streaming engine issues
its backward passes one at a time, so a single active slot suffices; a sink
is entered only around a backward call.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass

import torch

from thundersync_b200.ops.gemm import gemm_accumulate

_ACTIVE: "GradSink | None" = None

# CUDA: projection weight gradients (dW += dYᵀ·X into the sink) run on a side stream, so they fill the
# SMs that the dependent chain (dX, attention, norms) leaves idle; the stream that leaves a grad_sink
# block waits for them, so anything that reads the sink afterwards sees every deposit
SIDE_STREAM_WEIGHT_GRADS = True
_SIDE: dict[int, "torch.cuda.Stream"] = {}


def _side_stream(device: torch.device) -> "torch.cuda.Stream":
    idx = device.index if device.index is not None else torch.cuda.current_device()
    st = _SIDE.get(idx)
    if st is None:
        st = torch.cuda.Stream(device=idx)
        _SIDE[idx] = st
    return st


def active() -> "GradSink | None":
    return _ACTIVE


@contextlib.contextmanager
def grad_sink(sink: "GradSink | None"):
    global _ACTIVE
    prev = _ACTIVE
    _ACTIVE = sink
    try:
        yield sink
    finally:
        _ACTIVE = prev
        if sink is not None:
            sink.join_side_stream()


def _redirect_hook(p: torch.Tensor) -> None:
    s = _ACTIVE
    if s is None or p.grad is None or not s.owns(p):
        return
    g = p.grad
    p.grad = None
    s.add_(p, g)


def install_redirect_hooks(params) -> None:
    """Send gradients that autograd accumulates into ``param.grad`` to the active sink.

    Native ops deposit weight gradients into the sink themselves; parameters
    consumed by plain torch ops (decay logits, conv weights returned through
    autograd, adapters) reach ``AccumulateGrad`` instead. This hook moves such
    a contribution into the sink (with the sink's scale) the moment it lands.
    With no sink active it does nothing.
    """
    for p in params:
        if getattr(p, "_ts_redirect", False):
            continue
        p.register_post_accumulate_grad_hook(_redirect_hook)
        try:
            p._ts_redirect = True
        except Exception:
            pass


class ParamArena:
    """All trainable parameters re-homed into one contiguous flat buffer.

    Parameters keep their identity (``param.data`` becomes a view), so an
    optimizer built before or after adoption sees the same objects. Offsets
    are aligned to ``align`` elements; parameters registered back to back
    whose sizes are multiples of ``align`` stay adjacent, which lets
    q/k/v (and gate/up) run as one GEMM over a single weight view.
    """

    def __init__(self, params: list[torch.nn.Parameter], *, align: int = 64) -> None:
        seen: set[int] = set()
        uniq: list[torch.nn.Parameter] = []
        for p in params:
            if id(p) not in seen:
                seen.add(id(p))
                uniq.append(p)
        if not uniq:
            raise ValueError("a parameter arena needs at least one parameter")
        dtypes = {p.dtype for p in uniq}
        devices = {p.device for p in uniq}
        if len(dtypes) != 1 or len(devices) != 1:
            raise ValueError(f"arena parameters must share dtype and device, got {dtypes} {devices}")
        self.dtype = uniq[0].dtype
        self.device = uniq[0].device
        self.params = uniq
        self.offsets: dict[int, int] = {}
        off = 0
        for p in uniq:
            self.offsets[id(p)] = off
            off += -(-p.numel() // align) * align
        self.numel = off
        flat = torch.zeros(off, dtype=self.dtype, device=self.device)
        with torch.no_grad():
            for p in uniq:
                o = self.offsets[id(p)]
                view = flat[o : o + p.numel()].view_as(p)
                view.copy_(p.data)
                p.data = view
        self.flat = flat

    def owns(self, p: torch.Tensor) -> bool:
        return id(p) in self.offsets and p.data_ptr() == self.flat[self.offsets[id(p)] :].data_ptr()

    def rehome(self, flat: torch.Tensor) -> None:
        """Move every parameter into ``flat`` (same numel/dtype/device), keeping identity."""
        if flat.numel() < self.numel or flat.dtype != self.dtype or flat.device != self.device:
            raise ValueError("replacement arena buffer does not match")
        with torch.no_grad():
            flat[: self.numel].copy_(self.flat)
            for p in self.params:
                o = self.offsets[id(p)]
                p.data = flat[o : o + p.numel()].view_as(p)
        self.flat = flat[: self.numel]

    def resolve(self, t: torch.Tensor) -> torch.Tensor | None:
        """The arena parameter ``t`` is, or aliases exactly (same storage start and shape): activation
        checkpointing hands a recomputed backward detached aliases of the parameters it saved."""
        if id(t) in self.offsets:
            return t
        by_ptr = getattr(self, "_by_ptr", None)
        if by_ptr is None or getattr(self, "_by_ptr_flat", None) != self.flat.data_ptr():
            by_ptr = {p.data_ptr(): p for p in self.params}
            self._by_ptr, self._by_ptr_flat = by_ptr, self.flat.data_ptr()
        p = by_ptr.get(t.data_ptr()) if t.device == self.device else None
        return p if p is not None and p.shape == t.shape else None

    def offset(self, p: torch.Tensor) -> int:
        return self.offsets[id(p)]

    def view(self, buf: torch.Tensor, p: torch.Tensor) -> torch.Tensor:
        o = self.offsets.get(id(p))
        if o is None:
            q = self.resolve(p)
            if q is None:
                raise KeyError("tensor is not an arena parameter")
            o = self.offsets[id(q)]
        return buf[o : o + p.numel()].view(p.shape)

    def span(self, params: list[torch.Tensor]) -> tuple[int, int] | None:
        """(start, end) when ``params`` are exactly adjacent in the arena."""
        if not all(id(p) in self.offsets for p in params):
            return None
        start = self.offsets[id(params[0])]
        cur = start
        for p in params:
            if self.offsets[id(p)] != cur:
                return None
            cur += p.numel()
        return start, cur

    def fused_weight(self, params: list[torch.Tensor]) -> torch.Tensor | None:
        """One [sum(out), in] view over adjacent linear weights, else None."""
        sp = self.span(params)
        if sp is None or any(p.dim() != 2 or p.shape[1] != params[0].shape[1] for p in params):
            return None
        rows = sum(p.shape[0] for p in params)
        return self.flat[sp[0] : sp[1]].view(rows, params[0].shape[1])

    def new_buffer(self, dtype: torch.dtype = torch.float32, *, zero: bool = True) -> torch.Tensor:
        if zero:
            return torch.zeros(self.numel, dtype=dtype, device=self.device)
        return torch.empty(self.numel, dtype=dtype, device=self.device)


@dataclass
class GradSink:
    """Accumulate parameter gradients into ``buffer`` (fp32, arena layout).

    ``scale`` multiplies every deposited gradient (the reward-linear
    coefficient when a trajectory's advantage is already known).
    """

    arena: ParamArena
    buffer: torch.Tensor
    scale: float = 1.0
    deposits: int = 0

    def owns(self, p: torch.Tensor) -> bool:
        return id(p) in self.arena.offsets or self.arena.resolve(p) is not None

    def view(self, p: torch.Tensor) -> torch.Tensor:
        return self.arena.view(self.buffer, p)

    def span_view(self, params: list[torch.Tensor]) -> torch.Tensor | None:
        sp = self.arena.span(params)
        if sp is None:
            return None
        rows = sum(p.shape[0] for p in params)
        return self.buffer[sp[0] : sp[1]].view(rows, params[0].shape[1])

    def add_(self, p: torch.Tensor, grad: torch.Tensor) -> None:
        v = self.view(p)
        if self.scale != 1.0:
            v.add_(grad.to(v.dtype), alpha=self.scale)
        else:
            v.add_(grad)
        self.deposits += 1

    def addmm_(self, target: torch.Tensor, dy: torch.Tensor, x: torch.Tensor, *, side: bool = False) -> None:
        """``target += scale · dyᵀ x`` with fp32 accumulation, in place.

        ``side``: the caller guarantees no other deposit touches ``target`` before the sink block ends
        (a projection weight, which no native op or hook also writes), so on CUDA the GEMM may run on
        the side stream.
        """
        if dy.shape[0] == 0:
            return
        if target.is_cuda and dy.dtype != target.dtype:
            if side and SIDE_STREAM_WEIGHT_GRADS:
                main = torch.cuda.current_stream(target.device)
                st = _side_stream(target.device)
                st.wait_stream(main)
                with torch.cuda.stream(st):
                    gemm_accumulate(target, dy, x, a_t=True, b_t=False, alpha=self.scale)
                # the operands' memory must outlive the side-stream GEMM
                dy.record_stream(st)
                x.record_stream(st)
                self._side_devices = getattr(self, "_side_devices", set())
                self._side_devices.add(target.device)
            else:
                gemm_accumulate(target, dy, x, a_t=True, b_t=False, alpha=self.scale)
        else:
            target.addmm_(dy.t().to(target.dtype), x.to(target.dtype), alpha=self.scale)
        self.deposits += 1

    def join_side_stream(self) -> None:
        """Make the current stream wait for this sink's side-stream deposits."""
        devs = getattr(self, "_side_devices", None)
        if devs:
            for d in devs:
                torch.cuda.current_stream(d).wait_stream(_side_stream(d))
            devs.clear()
