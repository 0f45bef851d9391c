"""StreamingRun: one logical batch's streamed execution (C10-C18).

Events: ``open_group`` (forward the prompt once), ``append_turn`` /
``append_turns`` (forward each arriving turn over its trajectory's ancestor
chain, or only record it with ``stream_turns=False``), then the caller's
objective reads ``logprobs`` and backwards. The run produces per-trajectory
``log pi(token | context)`` and nothing else; it never sees a reward.

B200-first structure, in contrast to the reference's HF-hooked executor
(src/thundersync/engine/streaming.py:2974-7502):

* the model runs on :class:`~thundersync_b200.engine.layers.Executor`
  (native kernels, packed segments, one dense GEMM per projection per pack);
* per-layer K/V of every forwarded chunk are plain autograd tensors kept in
  each trajectory's chain: attention takes the chunk list directly, so
  retention is O(total tokens);
* with ``boundary_cut`` the prompt's outputs are cut by a
  :class:`~thundersync_b200.engine.boundary.Boundary` (detached proxy leaves
  with fp32 adjoint ledgers): a trajectory's backward stops at the prompt
  and the prompt is backwarded once per group;
* ``turn_boundary_rebuild`` cuts each turn's outgoing state the same way and
  replays the turns in reverse at trajectory close;
* trainable parameters live in one flat arena, so gradient sinks (fp32 flat
  buffers) can receive weight gradients straight from the GEMMs.

``old_logprobs(t)`` returns the detached twin of the exact tensor the update
backward flows through, so ``old == new`` holds bitwise.
"""

from __future__ import annotations

import contextlib
import time
import hashlib
from dataclasses import dataclass, field
from typing import Any, Callable, Iterable

import torch

from thundersync_b200.engine.boundary import Boundary
from thundersync_b200.engine.layers import Executor, Segment, executor_for
from thundersync_b200.ops.logprob import DEFAULT_ROWS, lm_head_logprob
from thundersync_b200.ops.sink import GradSink, ParamArena, grad_sink, install_redirect_hooks

__all__ = ["StreamingRun", "STREAM_ATTENTION_NAME", "register_stream_attention", "arena_for", "live_runs"]

STREAM_ATTENTION_NAME = "thundersync_stream"

_LIVE: "list[Any]" = []


PACK_ROW_MULTIPLE = 128


def register_stream_attention() -> None:
    """Kept for API compatibility with HF-hooked callers.

    This package's executor never calls a model's own attention function, so
    there is nothing to register: any Qwen3-structured model (this package's
    or HF's) runs through the native executor whatever its
    ``attn_implementation`` says.
    """
    return None


def live_runs() -> list["StreamingRun"]:
    import weakref  # noqa: F401

    return [r for r in _LIVE if r is not None]


def arena_for(model: torch.nn.Module) -> ParamArena | None:
    """The model's flat parameter arena (built once, rebuilt if stale)."""
    params = [p for p in model.parameters() if p.requires_grad]
    if not params:
        return None
    arena = getattr(model, "_ts_arena", None)
    if arena is not None:
        ids = {id(p) for p in params}
        if ids == set(arena.offsets) and all(arena.owns(p) for p in params):
            return arena
    dtypes = {p.dtype for p in params}
    devices = {p.device for p in params}
    if len(dtypes) != 1 or len(devices) != 1:
        return None
    arena = ParamArena(params)
    object.__setattr__(model, "_ts_arena", arena)
    return arena


@dataclass
class _Group:
    gid: int
    prompt: list[int]
    prompt_len: int
    chain: list[Any]  # per layer: ([k...], [v...]) or (tail, state) -- what branches read
    last: torch.Tensor  # hidden predicting the first turn token (proxy when cut)
    boundary: Boundary | None
    real_graph: list[torch.Tensor]
    trajs: list[int] = field(default_factory=list)
    shared_nodes: list[int] = field(default_factory=list)
    closed: bool = False


@dataclass
class _TurnCut:
    boundary: Boundary
    parent_chain: list[Any]
    parent_last: torch.Tensor
    tokens: list[int]
    pos0: int


@dataclass
class _Traj:
    tid: int
    gid: int
    chain: list[Any]
    last: torch.Tensor
    n_tokens: int
    turns: list[tuple[list[int], list[bool]]] = field(default_factory=list)
    logprobs: list[torch.Tensor] = field(default_factory=list)
    old: list[torch.Tensor] = field(default_factory=list)
    forwarded_turns: int = 0
    consumed_turns: int = 0
    cuts: list[_TurnCut] = field(default_factory=list)
    rebuilt: torch.Tensor | None = None
    rebuilt_old: torch.Tensor | None = None


@dataclass
class _SharedNode:
    idx: int
    tokens: list[int]
    parent: int | None
    groups: list[int]
    boundary: Boundary | None = None
    chain: list[Any] | None = None
    last: torch.Tensor | None = None
    pos_end: int = 0
    children: list[int] = field(default_factory=list)
    finalized: bool = False


def _flatten_state(states: list[Any], kinds: tuple[str, ...]) -> list[torch.Tensor]:
    out: list[torch.Tensor] = []
    for st, kind in zip(states, kinds):
        if st is None:
            continue
        for t in st:
            if isinstance(t, torch.Tensor):
                out.append(t)
    return out


def _rebuild_state(states: list[Any], flat: list[torch.Tensor]) -> list[Any]:
    it = iter(flat)
    out = []
    for st in states:
        if st is None:
            out.append(None)
            continue
        out.append(tuple(next(it) if isinstance(t, torch.Tensor) else t for t in st))
    return out


# Measured activations run a little above the per-token estimates (allocator rounding, fp32 row
# statistics); the memory rule scales its estimates by this factor.
TURN_ACTIVATION_FACTOR = 1.15


class StreamingRun:
    """One batch's streamed execution over a Qwen3-family model."""

    def __init__(
        self,
        model: torch.nn.Module,
        *,
        chunk: int | None = None,
        boundary_cut: bool = False,
        chunked_sdpa: bool = True,
        checkpoint: bool = False,
        stream_turns: bool = True,
        rebuild_block_tokens: int | None = 4096,
        rebuild_plain_reserve_bytes: int | None = None,
        prompt_checkpoint_storage_device: Any = None,
        rebuild_checkpoint_storage_device: Any = None,
        turn_boundary_rebuild: bool = False,
        boundary_adjoint_backend: str = "torch",
        boundary_adjoint_max_degree: int = 16,
        ragged_cohort_attention: bool = False,
        dependency_ready_shared_prefix_vjp: bool = False,
        shared_prefix_vjp_backend: str = "sequential",
        shared_prefix_vjp_timing: bool = False,
        shared_prefix_vjp_mode: str = "aggregate",
        explicit_adjoint_vjp: bool = False,
        parameter_adjoint_reduction: str = "arrival",
        parameter_adjoint_storage_device: Any = None,
    ) -> None:
        if getattr(model, "is_gradient_checkpointing", False):
            raise NotImplementedError(
                "HF gradient checkpointing is not supported; use StreamingRun(checkpoint=True)"
            )
        if turn_boundary_rebuild and not stream_turns:
            raise ValueError("turn-boundary rebuild requires stream_turns=True")
        if turn_boundary_rebuild and not boundary_cut:
            raise ValueError("turn-boundary rebuild requires boundary_cut=True")
        if turn_boundary_rebuild and model.training:
            raise ValueError("turn-boundary rebuild replays turns and requires model.eval()")
        if chunk is not None and chunk < 1:
            raise ValueError("chunk must be positive")
        if rebuild_block_tokens is not None and rebuild_block_tokens < 1:
            raise ValueError("rebuild_block_tokens must be positive or None")
        if boundary_adjoint_backend not in ("torch", "native", "triton"):
            raise ValueError("boundary_adjoint_backend must be torch or native (triton is accepted as a name for native)")
        if not 1 <= boundary_adjoint_max_degree <= 16:
            raise ValueError("boundary_adjoint_max_degree must be in [1, 16]")
        if shared_prefix_vjp_backend not in ("sequential", "ready_frontier", "isolated_canonical"):
            raise ValueError("unknown shared_prefix_vjp_backend")
        if shared_prefix_vjp_mode not in ("aggregate", "source_ready_serial"):
            raise ValueError("unknown shared_prefix_vjp_mode")
        if shared_prefix_vjp_backend == "isolated_canonical" or shared_prefix_vjp_mode == "source_ready_serial":
            from thundersync_b200.config import ConfigError

            raise ConfigError(
                "shared_prefix_vjp_backend='isolated_canonical' and shared_prefix_vjp_mode='source_ready_serial' "
                "are not built here (both keep per-node parameter contributions or graphs apart until the step): "
                "use 'sequential' or 'ready_frontier' with the 'aggregate' mode, and "
                "parameter_adjoint_reduction='canonical_source' for an order-independent sum")
        if parameter_adjoint_reduction not in ("arrival", "canonical_source"):
            raise ValueError("parameter_adjoint_reduction must be arrival or canonical_source")
        self.model = model
        self.chunk = DEFAULT_ROWS if chunk is None else int(chunk)  # LM-head rows per logits/dlogits block
        self.boundary_cut = boundary_cut
        self.chunked_sdpa = chunked_sdpa  # False: the concatenating baseline (see _retain_concatenated_chains)
        self.checkpoint = checkpoint
        self.stream_turns = stream_turns
        self.rebuild_block_tokens = rebuild_block_tokens
        self.turn_boundary_rebuild = turn_boundary_rebuild
        self.boundary_adjoint_backend = boundary_adjoint_backend
        self.boundary_adjoint_max_degree = boundary_adjoint_max_degree
        # every boundary ledger sums its consumers' adjoints with this backend (engine/boundary.py)
        self._boundary_kw = {"reduce_backend": boundary_adjoint_backend, "max_degree": boundary_adjoint_max_degree}
        self.parameter_adjoint_reduction = parameter_adjoint_reduction
        self.shared_prefix_vjp_mode = shared_prefix_vjp_mode
        self.explicit_adjoint_vjp = bool(explicit_adjoint_vjp)
        self.shared_prefix_vjp_backend = shared_prefix_vjp_backend
        self.shared_prefix_vjp_timing = bool(shared_prefix_vjp_timing)
        self._shared_prefix_times: list[float] = []
        # set by objectives whose unscored turns have no loss of their own (on-policy distillation turns)
        self.defer_unscored_turns = False
        self._deferred_turns = 0  # turns held back at arrival
        self._deferred_forwards = 0  # held-back turns forwarded when a later turn needed their state
        self._shared_prefix_calls = 0  # autograd calls over shared prompt nodes
        self._shared_prefix_early = 0  # nodes run before the batch barrier (dependency-ready)
        # staged parameter adjoints (canonical-source reduction) live here until they are applied
        self._param_adjoint_device = (
            None if parameter_adjoint_storage_device is None else torch.device(parameter_adjoint_storage_device)
        )
        self.rebuild_plain_reserve_bytes = rebuild_plain_reserve_bytes
        self.dependency_ready_shared_prefix_vjp = dependency_ready_shared_prefix_vjp or (
            shared_prefix_vjp_mode == "source_ready_serial"
        )
        self._rebuild_checkpoint_storage_device = (
            None if rebuild_checkpoint_storage_device is None else torch.device(rebuild_checkpoint_storage_device)
        )
        self.device = next(model.parameters()).device
        self.arena = arena_for(model)
        self.exec: Executor = executor_for(model, self.arena)
        self.spec = self.exec.spec
        self.weight = self.exec.head_weight()
        self._groups: dict[int, _Group] = {}
        self._trajs: dict[int, _Traj] = {}
        self._traj_group: dict[int, int] = {}
        self._shared: list[_SharedNode] = []
        self._trainable = [p for p in model.parameters() if p.requires_grad]
        install_redirect_hooks(self._trainable)
        self._versions = {id(p): p._version for p in self._trainable}
        self._capture_source: Any = None
        self._param_adjoint_staged: dict[Any, list[tuple[torch.Tensor, torch.Tensor]]] = {}
        self._counts = {"plain": 0, "blocked": 0, "checkpoint": 0, "checkpoint_host": 0, "turn_forward": 0,
                        "turn_replay": 0, "prompt_forward": 0}
        self._turn_counts: dict[str, dict[str, int]] = {"forward": {}, "replay": {}}
        self._prompt_tokens_physical = 0
        self._prompt_tokens_logical = 0
        self._last_rung: str | None = None
        self._pack_rung: str | None = None  # the rebuild rung a pack runs under (None: not a close rebuild)
        self._offload = {"write_bytes": 0, "read_bytes": 0, "tensors": 0}
        self._oom_retries = 0
        self._memory_windows: list[dict[str, Any]] = []
        self._memory_window: dict[str, Any] | None = None
        self._memory_refusals: dict[str, int] = {}
        self._memory_min_available: int | None = None
        self._memory_retries_at_start: int | None = None
        _LIVE.append(self)

    # ------------------------------------------------------------ helpers
    def _ids(self, values: Iterable[int]) -> torch.Tensor:
        """Token ids on the run's device, copied from page-locked host memory."""
        if isinstance(values, torch.Tensor):
            t = values.to(dtype=torch.long).reshape(-1)
            if t.device == self.device:
                return t
        else:
            t = torch.tensor(list(values), dtype=torch.long)
        if self.device.type == "cuda":
            if not t.is_pinned():
                t = t.pin_memory()
            return t.to(self.device, non_blocking=True)
        return t.to(self.device)

    def _positions(self, start: int, n: int) -> torch.Tensor:
        return torch.arange(start, start + n, dtype=torch.long, device=self.device)

    def _run_pack(self, ids: torch.Tensor, pos: torch.Tensor, segs: list[Segment]):
        # On CUDA the pack's row count is padded to a multiple of PACK_ROW_MULTIPLE
        # (token 0 at position 0; no segment covers those rows, so they receive no
        # attention, produce no state and get zero gradient): every GEMM then
        # sees one of a few dozen shapes, and the library's per-shape algorithm
        # selection, which costs hundreds of microseconds of host time for a new
        # shape, is paid once per shape instead of once per trajectory.
        t = ids.shape[0]
        pad = (-t) % PACK_ROW_MULTIPLE if ids.is_cuda else 0
        if pad:
            ids = torch.cat((ids, ids.new_zeros(pad)))
            pos = torch.cat((pos, pos.new_zeros(pad)))
        rung = self._pack_rung
        if torch.is_grad_enabled() and (self.checkpoint or rung in ("checkpoint", "checkpoint_host")):
            host = rung == "checkpoint_host" or (rung is not None and self._rebuild_checkpoint_storage_device
                                                 is not None and self._rebuild_checkpoint_storage_device.type == "cpu")
            with (self._checkpoint_inputs_on_host() if host else contextlib.nullcontext()):
                h, states = self._run_pack_checkpointed(ids, pos, segs)
        else:
            h, states = self.exec.run(ids, pos, segs)
        if not self.chunked_sdpa and h.grad_fn is not None:
            self._retain_concatenated_chains(h, segs, states)
        return (h[:t] if pad else h), states

    def _retain_concatenated_chains(self, h: torch.Tensor, segs: list[Segment], states: list[Any]) -> None:
        """``chunked_sdpa=False``: keep, for as long as this pack's graph lives, each segment's concatenated
        [ancestors | own] key/value chain per attention layer -- what a concatenate-then-attend op saves for
        its backward. The streamed path never does this; the mode exists as the baseline that the memory
        regression gate measures it against."""
        keep = []
        for seg, st in zip(segs, states):
            for i in self.spec.attention_layers:
                past = seg.past[i] if seg.past and seg.past[i] is not None else ([], [])
                own = st[i]
                keep.append(torch.cat([*past[0], own[0]], 0))
                keep.append(torch.cat([*past[1], own[1]], 0))
        h.grad_fn.metadata["concatenated_chains"] = keep

    @contextlib.contextmanager
    def _checkpoint_inputs_on_host(self):
        """Park the tensors autograd saves in this forward (the per-layer checkpoint inputs) in page-locked
        host memory until the backward needs them; counts the bytes each way."""
        diag = self._offload

        def pack(t: torch.Tensor):
            if t.device.type != "cuda" or t.numel() * t.element_size() < 1 << 16:
                return t  # small tensors (norm weights, scalars) stay where they are
            host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            host.copy_(t, non_blocking=True)
            diag["write_bytes"] += host.numel() * host.element_size()
            diag["tensors"] += 1
            return (t.device, host)

        def unpack(obj):
            if isinstance(obj, torch.Tensor):
                return obj
            dev, host = obj
            diag["read_bytes"] += host.numel() * host.element_size()
            return host.to(dev, non_blocking=True)

        with torch.autograd.graph.saved_tensors_hooks(pack, unpack):
            yield

    def _run_pack_checkpointed(self, ids, pos, segs):
        """Per-layer activation checkpointing; fresh K/V are checkpoint outputs."""
        from torch.utils.checkpoint import checkpoint

        ex = self.exec
        h = ex.embed(ids)
        states: list[list[Any]] = [[None] * ex.spec.n_layers for _ in segs]
        for i, kind in enumerate(ex.spec.kinds):
            fn = ex.attention_layer if kind == "full_attention" else ex.linear_layer

            def body(h_in, _i=i, _fn=fn):
                h_out, new = _fn(_i, h_in, pos, segs)
                flat = [t for st in new for t in st if isinstance(t, torch.Tensor)]
                return (h_out, *flat)

            outs = checkpoint(body, h, use_reentrant=False)
            h = outs[0]
            it = iter(outs[1:])
            for j in range(len(segs)):
                states[j][i] = (next(it), next(it))
        return ex.final_norm(h), states

    def _check_versions(self) -> None:
        for p in self._trainable:
            if p._version != self._versions.get(id(p), p._version):
                raise RuntimeError(
                    "a trainable parameter changed inside a logical batch; parameters must "
                    "stay fixed until assert_safe_to_step() and the optimizer step"
                )

    def _chain_extend(self, chain: list[Any], states: list[Any]) -> list[Any]:
        out = []
        for kind, base, st in zip(self.spec.kinds, chain, states):
            if kind == "full_attention":
                ks, vs = base if base is not None else ([], [])
                out.append(([*ks, st[0]], [*vs, st[1]]))
            else:
                out.append(st)
        return out

    def _scored_logprobs(self, hs: torch.Tensor, last: torch.Tensor, tokens: list[int], scored: list[bool]):
        """Predecessor rows of the scored tokens -> fp32 log-probs (graph-attached)."""
        idx = [j for j, s in enumerate(scored) if s]
        if not idx:
            return hs.new_zeros(0, dtype=torch.float32)
        rows = torch.cat((last[None], hs[:-1]), 0) if hs.shape[0] > 0 else last[None]
        tgt = self._ids([tokens[j] for j in idx])
        if idx[-1] - idx[0] + 1 == len(idx):  # one contiguous run (every completion token scored): a view
            picked = rows[idx[0]:idx[-1] + 1]
        else:  # index copied from page-locked memory: no host wait on the device queue
            picked = rows.index_select(0, self._ids(idx))
        return lm_head_logprob(picked, self.weight, tgt, rows=self.chunk)

    # ------------------------------------------------------------ groups
    def open_group(self, group_id: int, prompt_tokens: list[int]) -> None:
        if group_id in self._groups:
            raise ValueError(f"group {group_id} is already open")
        prompt = [int(t) for t in prompt_tokens]
        if not prompt:
            raise ValueError("a prompt must contain at least one token")
        self._check_versions()
        ids = self._ids(prompt)
        pos = self._positions(0, len(prompt))
        h, states = self._run_pack(ids, pos, [Segment(0, len(prompt), [])])
        self._counts["prompt_forward"] += 1
        self._prompt_tokens_physical += len(prompt)
        self._prompt_tokens_logical += len(prompt)
        st = states[0]
        chain = self._chain_extend([None] * self.spec.n_layers, st)
        self._install_group(group_id, prompt, chain, h[-1])

    def _install_group(self, gid: int, prompt: list[int], chain: list[Any], last: torch.Tensor, shared=()):
        real_flat = _flatten_chain(chain) + [last]
        boundary = None
        if self.boundary_cut and last.requires_grad:
            boundary = Boundary.cut(real_flat, capture_source=lambda: self._capture_source, **self._boundary_kw)
            flat = boundary.proxy
            chain = _unflatten_chain(chain, flat[:-1])
            last = flat[-1]
        self._groups[gid] = _Group(
            gid=gid, prompt=prompt, prompt_len=len(prompt), chain=chain, last=last,
            boundary=boundary, real_graph=real_flat, shared_nodes=list(shared),
        )

    def open_groups_shared_prefix(self, groups: dict[int, list[int]] | list[tuple[int, list[int]]]) -> None:
        """Open several groups whose prompts share token prefixes (a radix prompt forest).

        Each shared prefix node is forwarded once; with ``boundary_cut`` it is
        cut like a prompt and backwarded once, after its last consumer group
        closed, by :meth:`finalize_shared_prefixes` (reference:
        src/thundersync/engine/streaming.py:3444-3768).
        """
        items = list(groups.items()) if isinstance(groups, dict) else list(groups)
        for gid, _ in items:
            if gid in self._groups:
                raise ValueError(f"group {gid} is already open")
        self._check_versions()
        prompts = {gid: [int(t) for t in p] for gid, p in items}
        # radix split over group prompts
        nodes: list[_SharedNode] = []
        leaf_parent: dict[int, int | None] = {}
        leaf_offset: dict[int, int] = {}

        def split(gids: list[int], offset: int, parent: int | None) -> None:
            if len(gids) == 1:
                leaf_parent[gids[0]] = parent
                leaf_offset[gids[0]] = offset
                return
            seqs = [prompts[g][offset:] for g in gids]
            lo, hi = 0, min(len(s) for s in seqs)
            while lo < hi:
                mid = (lo + hi + 1) // 2
                if all(s[:mid] == seqs[0][:mid] for s in seqs[1:]):
                    lo = mid
                else:
                    hi = mid - 1
            share = lo
            node_parent = parent
            if share > 0:
                node = _SharedNode(len(self._shared) + len(nodes), seqs[0][:share], parent, list(gids))
                nodes.append(node)
                node_parent = node.idx
                if parent is not None:
                    self._node(parent, nodes).children.append(node.idx)
            buckets: dict[Any, list[int]] = {}
            for g in gids:
                rest = prompts[g][offset + share :]
                key = rest[0] if rest else None
                buckets.setdefault(key, []).append(g)
            for key, members in buckets.items():
                if key is None or len(members) == 1:
                    for g in members:
                        leaf_parent[g] = node_parent
                        leaf_offset[g] = offset + share
                else:
                    split(members, offset + share, node_parent)

        split(sorted(prompts), 0, None)
        self._shared.extend(nodes)
        # forward shared nodes parent-first
        for node in nodes:
            base_chain, base_last, pos0 = self._node_context(node.parent)
            ids = self._ids(node.tokens)
            segs = [Segment(0, len(node.tokens), base_chain)]
            h, states = self._run_pack(ids, self._positions(pos0, len(node.tokens)), segs)
            self._prompt_tokens_physical += len(node.tokens)
            chain = self._chain_extend(base_chain, _own_only(states[0]))
            last = h[-1]
            own_real = _flatten_state(states[0], self.spec.kinds) + [last]
            if self.boundary_cut and last.requires_grad:
                node.boundary = Boundary.cut(own_real, capture_source=lambda: self._capture_source,
                                             **self._boundary_kw)
                prox = node.boundary.proxy
                chain = self._chain_replace_tail(chain, base_chain, prox[:-1])
                last = prox[-1]
            node.chain, node.last, node.pos_end = chain, last, pos0 + len(node.tokens)
        # each group's own suffix
        for gid, prompt in prompts.items():
            parent = leaf_parent[gid]
            base_chain, base_last, pos0 = self._node_context(parent)
            suffix = prompt[leaf_offset[gid] :]
            self._prompt_tokens_logical += len(prompt)
            shared_ids = self._ancestor_nodes(parent)
            if suffix:
                h, states = self._run_pack(
                    self._ids(suffix), self._positions(pos0, len(suffix)), [Segment(0, len(suffix), base_chain)]
                )
                self._prompt_tokens_physical += len(suffix)
                chain = self._chain_extend(base_chain, states[0])
                last = h[-1]
            else:
                chain, last = base_chain, base_last
            self._install_group(gid, prompt, chain, last, shared=shared_ids)
            self._counts["prompt_forward"] += 1

    def _node(self, idx: int, pending: list[_SharedNode] | None = None) -> _SharedNode:
        if idx < len(self._shared):
            return self._shared[idx]
        assert pending is not None
        return pending[idx - len(self._shared)]

    def _node_context(self, idx: int | None):
        if idx is None:
            return [None] * self.spec.n_layers, None, 0
        node = self._shared[idx] if idx < len(self._shared) else None
        assert node is not None and node.chain is not None
        return node.chain, node.last, node.pos_end

    def _ancestor_nodes(self, idx: int | None) -> list[int]:
        out = []
        while idx is not None:
            out.append(idx)
            idx = self._shared[idx].parent
        return out

    def _chain_replace_tail(self, chain, base_chain, flat_tail: list[torch.Tensor]):
        """Replace the tensors appended on top of ``base_chain`` by ``flat_tail``."""
        it = iter(flat_tail)
        out = []
        for kind, full, base in zip(self.spec.kinds, chain, base_chain):
            if kind == "full_attention":
                ks, vs = full
                nb = 0 if base is None else len(base[0])
                ks = list(ks[:nb]) + [next(it) for _ in ks[nb:]]
                vs = list(vs[:nb]) + [next(it) for _ in vs[nb:]]
                out.append((ks, vs))
            else:
                out.append(tuple(next(it) if isinstance(t, torch.Tensor) else t for t in full))
        return out

    def boundary(self, group_id: int) -> Boundary:
        b = self._groups[group_id].boundary
        if b is None:
            raise RuntimeError("this run has no boundary cut")
        return b

    def group_of(self, traj_id: int) -> int:
        return self._traj_group[traj_id]

    def open_group_ids(self) -> list[int]:
        return [g for g, st in self._groups.items() if not st.closed]

    def trajectories_of(self, group_id: int) -> list[int]:
        return list(self._groups[group_id].trajs)

    # ------------------------------------------------------------ turns
    def _check_traj(self, group_id: int, traj_id: int) -> None:
        """Raise if a turn of ``traj_id`` in ``group_id`` cannot be recorded (changes nothing)."""
        t = self._trajs.get(traj_id)
        if t is None:
            g = self._groups.get(group_id)
            if g is None or g.closed:
                raise KeyError(f"group {group_id} is not open")
            if traj_id in self._traj_group:
                raise ValueError(f"trajectory {traj_id} was already freed")
        elif t.gid != group_id:
            raise ValueError(f"trajectory {traj_id} belongs to group {t.gid}, not {group_id}")

    def _traj_state(self, group_id: int, traj_id: int) -> _Traj:
        self._check_traj(group_id, traj_id)
        t = self._trajs.get(traj_id)
        if t is None:
            g = self._groups[group_id]
            t = _Traj(tid=traj_id, gid=group_id, chain=g.chain, last=g.last, n_tokens=g.prompt_len)
            self._trajs[traj_id] = t
            self._traj_group[traj_id] = group_id
            g.trajs.append(traj_id)
        return t

    def append_turn(self, group_id: int, traj_id: int, tokens: list[int], scored: list[bool]) -> None:
        self.append_turns([(group_id, traj_id, tokens, scored)])

    def append_turns(self, items: list[tuple[int, int, list[int], list[bool]]], *, joint_backward: bool = False) -> None:
        """Record (and with ``stream_turns``, forward) arriving turns.

        ``joint_backward``: the caller backwards the losses of these turns together (one backward per
        call, as the scored-turn packs of on-policy distillation do), so several trajectories may forward
        as one pack. Otherwise every trajectory's turn forwards on its own: a per-trajectory backward
        through a shared pack graph would free the pack's saved tensors under the other trajectories.
        Every item is checked before any state changes."""
        checked = []
        for gid, tid, tokens, scored in items:
            tokens = [int(t) for t in tokens]
            scored = [bool(s) for s in scored]
            if len(tokens) != len(scored):
                raise ValueError("tokens and scored mask must have equal length")
            if not tokens:
                raise ValueError("a turn must contain at least one token")
            self._check_traj(gid, tid)
            checked.append((gid, tid, tokens, scored))
        pending: list[tuple[_Traj, list[int], list[bool], int]] = []  # (trajectory, tokens, scored, turn index)
        for gid, tid, tokens, scored in checked:
            t = self._traj_state(gid, tid)
            t.turns.append((tokens, scored))
            pending.append((t, tokens, scored, len(t.turns) - 1))
        if not self.stream_turns:
            for t, tokens, _, _ in pending:
                t.n_tokens += len(tokens)
            return
        self._check_versions()
        # a trajectory appearing twice in one call forwards in rounds; with a turn memory rule a joint
        # round runs as the widest leading packs the device admits (joint_turn_pack_width)
        while pending:
            seen: set[int] = set()
            this, rest = [], []
            for item in pending:
                (rest if item[0].tid in seen else this).append(item)
                seen.add(item[0].tid)
            if self.defer_unscored_turns:
                this = self._settle_deferred(this)
            while this:
                width = 1
                if joint_backward and len(this) > 1:
                    width = self.joint_turn_pack_width([(t.gid, t.tid, tokens, scored)
                                                        for t, tokens, scored, _ in this])
                    if not self.joint_turn_pack_ready:
                        width = len(this)  # without turn-boundary replay a joint round is one pack
                self._forward_turns([x[:3] for x in this[:width]])
                this = this[width:]
            pending = rest

    # ------------------------------------------------------------ joint turn packs
    def _joint_conditions(self) -> bool:
        # a joint pack's one backward belongs to several trajectories: the parameter adjoints must
        # accumulate in arrival order (no per-source reduction, no per-source serial drain, no explicit
        # per-source VJP), the turns' outgoing state must be cut for replay, and every layer must be an
        # attention layer (a linear-attention state carries no per-segment boundary here)
        return (self.stream_turns and self.turn_boundary_rebuild and self.chunked_sdpa
                and all(k == "full_attention" for k in self.spec.kinds)
                and self.parameter_adjoint_reduction != "canonical_source"
                and self.shared_prefix_vjp_mode != "source_ready_serial"
                and not self.explicit_adjoint_vjp)

    @property
    def joint_turn_pack_ready(self) -> bool:
        """Whether several ready turns may forward as one plain, jointly backwarded pack (reference:
        src/thundersync/engine/streaming.py:3898-3919)."""
        return self._joint_conditions()

    @property
    def joint_turn_replay_ready(self) -> bool:
        """Whether the turn replays of several closed trajectories may run as one joint pack (same
        conditions as :attr:`joint_turn_pack_ready`)."""
        return self._joint_conditions()

    def _turn_pack_estimate(self, tokens: int, past_tokens: int) -> int:
        """Peak bytes a plain pack of ``tokens`` new tokens over ``past_tokens`` ancestor rows keeps."""
        shape = self._turn_memory_shape()
        return tokens * (shape["plain_activation"] + shape["kv"] + 2 * shape["hidden"]) + past_tokens * shape["kv"]

    def _pack_fits(self, needs: list[tuple[int, int]], avail: int | None) -> bool:
        if avail is None:
            return True
        tokens = sum(n for n, _ in needs)
        past = sum(p for _, p in needs)
        return self._turn_pack_estimate(tokens, past) + (self.rebuild_plain_reserve_bytes or 0) <= avail

    def joint_turn_pack_width(self, items: list[tuple[int, int, list[int], list[bool]]]) -> int:
        """How many leading turns of ``items`` one plain joint pack carries (reference:
        src/thundersync/engine/streaming.py:3921-3955): every turn without the checkpoint flag (full
        activations are retained by construction); with it, the widest prefix whose estimated peak plus
        ``rebuild_plain_reserve_bytes`` fits the memory available now (read once), else 1."""
        if len(items) < 2 or not self.joint_turn_pack_ready:
            return 1
        if not self.checkpoint:
            return len(items)
        if self.rebuild_plain_reserve_bytes is None:
            return 1
        avail = self._available_bytes() if self.device.type == "cuda" else None
        needs = []
        for gid, tid, tokens, _ in items:
            t = self._trajs.get(tid)  # n_tokens: the turn's first position (prompt included)
            past = t.n_tokens if t is not None else (self._groups[gid].prompt_len if gid in self._groups else 0)
            needs.append((len(tokens), past))
        for width in range(len(items), 1, -1):
            if self._pack_fits(needs[:width], avail):
                if width < len(items):
                    self._memory_refusals["pack_narrowed"] = self._memory_refusals.get("pack_narrowed", 0) + 1
                return width
        self._memory_refusals["pack_refused"] = self._memory_refusals.get("pack_refused", 0) + 1
        return 1

    def _turn_replay_pack(self, needs: list[tuple[int, int]]) -> list[int]:
        """Which of the ready replays (one per cohort member, in order) one model call carries: each joins
        while the pack's estimate plus the reserve fits; fewer than two admitted is no pack ([0])."""
        if len(needs) < 2 or not self.joint_turn_replay_ready:
            return [0]
        if not self.checkpoint:
            return list(range(len(needs)))
        if self.rebuild_plain_reserve_bytes is None:
            return [0]
        avail = self._available_bytes() if self.device.type == "cuda" else None
        chosen: list[int] = []
        for i, need in enumerate(needs):
            if self._pack_fits([needs[j] for j in chosen] + [need], avail):
                chosen.append(i)
        return chosen if len(chosen) >= 2 else [0]

    def trajectory_tokens(self, traj_id: int) -> int:
        """Tokens of a trajectory's own branch (its turns, not the shared prompt)."""
        t = self._trajs[traj_id]
        return sum(len(tk) for tk, _ in t.turns)

    def _settle_deferred(self, items: list[tuple[_Traj, list[int], list[bool], int]]):
        """With ``defer_unscored_turns``: before a trajectory's new turn forwards, its deferred turns
        forward first, each as its own single-turn call at its own positions; a new turn without a
        scored token is itself deferred (its state is read only by a later turn of its trajectory, and a
        turn that ends the trajectory is never forwarded). Returns the items to forward now."""
        out = []
        for item in items:
            t, _, scored, k = item
            while t.forwarded_turns < k:
                tk, sc = t.turns[t.forwarded_turns]
                self._forward_turns([(t, tk, sc)])
                self._deferred_forwards += 1
            if any(scored):
                out.append(item)
            else:
                self._deferred_turns += 1
        return out

    def forward_deferred_turns(self, traj_id: int) -> None:
        t = self._trajs[traj_id]
        if t.forwarded_turns < len(t.turns):
            todo = t.turns[t.forwarded_turns :]
            for tokens, scored in todo:
                self._forward_turns([(t, tokens, scored)])

    def _forward_turns(self, items: list[tuple[_Traj, list[int], list[bool]]]) -> None:
        ids, pos, segs = [], [], []
        cur = 0
        for t, tokens, _ in items:
            ids.extend(tokens)
            pos.append(self._positions(t.n_tokens, len(tokens)))
            segs.append(Segment(cur, len(tokens), t.chain))
            cur += len(tokens)
        h, states = self._run_pack(self._ids(ids), torch.cat(pos), segs)
        self._counts["turn_forward"] += 1
        key = str(len(items))
        self._turn_counts["forward"][key] = self._turn_counts["forward"].get(key, 0) + 1
        for (t, tokens, scored), seg, st in zip(items, segs, states):
            hs = h[seg.start : seg.start + seg.length]
            lp = self._scored_logprobs(hs, t.last, tokens, scored)
            t.logprobs.append(lp)
            t.old.append(lp.detach())
            pos0 = t.n_tokens
            chain = self._chain_extend(t.chain, st)
            last = hs[-1]
            if self.turn_boundary_rebuild:
                own = _flatten_state(st, self.spec.kinds) + [last]
                b = Boundary.cut(own, capture_source=lambda: self._capture_source, **self._boundary_kw)
                b.real = [x.detach() for x in b.real]  # replay re-forwards; keep no graph
                t.cuts.append(_TurnCut(b, t.chain, t.last, tokens, pos0))
                chain = self._chain_replace_tail(chain, t.chain, b.proxy[:-1])
                last = b.proxy[-1]
            t.chain = chain
            t.last = last
            t.n_tokens += len(tokens)
            t.forwarded_turns += 1

    # ------------------------------------------------------------ logprobs
    def logprobs(self, traj_id: int, *, rebuild: bool = False) -> torch.Tensor:
        t = self._trajs[traj_id]
        if rebuild or not self.stream_turns:
            if t.rebuilt is None or rebuild:
                self.rebuild_logprobs([traj_id])
            return t.rebuilt
        if not t.logprobs:
            return torch.zeros(0, dtype=torch.float32, device=self.device)
        return t.logprobs[0] if len(t.logprobs) == 1 else torch.cat(t.logprobs)

    def old_logprobs(self, traj_id: int) -> torch.Tensor:
        t = self._trajs[traj_id]
        if not self.stream_turns or t.rebuilt_old is not None:
            if t.rebuilt_old is None:
                raise RuntimeError(
                    "with stream_turns=False old log-probs are defined by the close rebuild; "
                    "call logprobs(..., rebuild=True) or rebuild_logprobs first"
                )
            return t.rebuilt_old
        if not t.old:
            return torch.zeros(0, dtype=torch.float32, device=self.device)
        return t.old[0] if len(t.old) == 1 else torch.cat(t.old)

    def consume_latest_turn_logprobs(self, traj_id: int) -> tuple[torch.Tensor, torch.Tensor]:
        t = self._trajs[traj_id]
        if t.forwarded_turns < len(t.turns):  # the latest turn is deferred: it has no log-probs yet
            empty = torch.zeros(0, dtype=torch.float32, device=self.device)
            return empty, empty
        if not t.logprobs:
            raise RuntimeError("no forwarded turn to consume")
        lp, old = t.logprobs[-1], t.old[-1]
        t.logprobs[-1] = lp.detach()
        t.consumed_turns = t.forwarded_turns
        return lp, old

    # ------------------------------------------------------------ memory rule
    REBUILD_RUNGS = ("plain", "blocked", "checkpoint", "checkpoint_host")

    def _turn_memory_shape(self) -> dict[str, int]:
        """Bytes per token that a forward keeps for the backward, by executor (estimates)."""
        sp = self.spec
        el = self.weight.element_size()
        hidden = sp.hidden
        kv = 2 * sp.n_kv * sp.head_dim * el * len(sp.attention_layers)  # retained K and V rows
        # per layer: normed input, q/k/v, attention output, residual, normed input, gate/up and their
        # product, plus fp32 row statistics -- about 16 hidden-width rows in the activation dtype
        plain = sp.n_layers * hidden * el * 16
        checkpoint = sp.n_layers * hidden * el + hidden * el * 16  # layer inputs + one layer recomputed
        return {"plain_activation": int(plain * TURN_ACTIVATION_FACTOR),
                "checkpoint_activation": int(checkpoint * TURN_ACTIVATION_FACTOR),
                "host_checkpoint_activation": int(hidden * el * 16 * TURN_ACTIVATION_FACTOR),
                "kv": kv, "hidden": hidden * el}

    def _available_bytes(self) -> int:
        free, _ = torch.cuda.mem_get_info(self.device)
        cached = torch.cuda.memory_reserved(self.device) - torch.cuda.memory_allocated(self.device)
        avail = int(free + max(cached, 0))
        self._memory_min_available = avail if self._memory_min_available is None else min(
            self._memory_min_available, avail)
        return avail

    def _rung_estimate(self, rung: str, tokens: int) -> int:
        shape = self._turn_memory_shape()
        key = {"plain": "plain_activation", "blocked": "plain_activation", "checkpoint": "checkpoint_activation",
               "checkpoint_host": "host_checkpoint_activation"}[rung]
        return tokens * (shape[key] + shape["kv"] + 2 * shape["hidden"])

    def _choose_rung(self, tokens: int, *, extra: int = 0) -> str:
        """The first rung whose estimate fits the device beside the configured reserve (``extra``: bytes the
        caller frees before the backward, counted as available)."""
        if self.device.type != "cuda":
            return "checkpoint" if self.checkpoint else "blocked"
        reserve = self.rebuild_plain_reserve_bytes or 0
        avail = self._available_bytes() + max(0, extra)
        first = 2 if self.checkpoint else 0
        for rung in self.REBUILD_RUNGS[first:]:
            if rung == "plain" and self.rebuild_plain_reserve_bytes is None:
                continue  # without a reserve the automatic rebuild starts blocked (bounded transient)
            if self._rung_estimate(rung, tokens) + reserve <= avail:
                return rung
            self._memory_refusals[rung] = self._memory_refusals.get(rung, 0) + 1
        return "checkpoint_host"

    def _open_memory_window(self, phase: str, executor: str, estimate: int) -> None:
        if self.device.type != "cuda":
            return
        self.close_memory_window()
        if self._memory_retries_at_start is None:
            self._memory_retries_at_start = int(torch.cuda.memory_stats(self.device).get("num_alloc_retries", 0))
        torch.cuda.reset_peak_memory_stats(self.device)
        self._memory_window = {"phase": phase, "executor": executor, "estimate": int(estimate),
                               "allocated": int(torch.cuda.memory_allocated(self.device))}

    def rebuild_logprobs(
        self,
        traj_ids: list[int],
        *,
        joint_backward: bool = False,
        executor: str = "auto",
        checkpoint_input_storage_device: Any = None,
        releasing_bytes: int | Callable[[], int] | None = None,
    ) -> list[torch.Tensor]:
        """Re-forward whole branches (all turns) over the prompt chain.

        With ``joint_backward`` (the caller backwards the branches' log-probs together) several branches
        forward as one pack; otherwise each branch forwards on its own, so that one branch's backward
        never frees a graph another branch still needs. ``releasing_bytes`` (bytes, or a callable giving
        them) is device memory the caller frees before the backward: the automatic rung choice counts it
        as available.

        ``executor`` picks the rung of the memory ladder: ``plain`` (one pack per call, every activation
        kept), ``blocked`` (branches longer than ``rebuild_block_tokens`` run in consecutive blocks, each
        attending to the previous blocks' K/V, so the transient stays block-sized), ``checkpoint``
        (per-layer activation checkpointing: only layer inputs are kept), ``checkpoint_host`` (those
        inputs wait in page-locked host memory). ``auto`` takes the first rung whose estimate fits the
        device beside ``rebuild_plain_reserve_bytes`` and, when a forward still runs out of device memory,
        frees what it built and retries one rung lower. ``checkpoint_input_storage_device="cpu"`` makes
        the checkpoint rungs park their inputs on the host.
        """
        rungs = ("auto", *self.REBUILD_RUNGS)
        if executor not in rungs:
            raise ValueError(f"executor must be one of {rungs}")
        self._check_versions()
        if len(traj_ids) > 1 and not joint_backward:
            return [self.rebuild_logprobs([t], executor=executor, releasing_bytes=releasing_bytes,
                                          checkpoint_input_storage_device=checkpoint_input_storage_device)[0]
                    for t in traj_ids]
        trajs = [self._trajs[t] for t in traj_ids]
        n_tok = sum(len(x) for t in trajs for x, _ in t.turns)
        if executor != "auto":
            rung = executor
        else:
            extra = releasing_bytes() if callable(releasing_bytes) else (releasing_bytes or 0)
            rung = self._choose_rung(n_tok, extra=int(extra))
        if checkpoint_input_storage_device is not None and torch.device(checkpoint_input_storage_device).type == "cpu" \
                and rung == "checkpoint":
            rung = "checkpoint_host"
        while True:
            try:
                self._open_memory_window("rebuild", rung, self._rung_estimate(rung, n_tok))
                return self._rebuild_at(trajs, rung)
            except torch.cuda.OutOfMemoryError:
                nxt = self.REBUILD_RUNGS.index(rung) + 1
                if executor != "auto" or nxt >= len(self.REBUILD_RUNGS):
                    raise
                for t in trajs:
                    t.rebuilt = t.rebuilt_old = None
                self._memory_window = None
                torch.cuda.empty_cache()
                self._oom_retries += 1
                rung = self.REBUILD_RUNGS[nxt]
            finally:
                self._pack_rung = None

    def _rebuild_at(self, trajs: list[_Traj], rung: str) -> list[torch.Tensor]:
        block = self.rebuild_block_tokens if rung != "plain" else None
        self._pack_rung = rung
        toks = []
        masks = []
        for t in trajs:
            tk = [x for tokens, _ in t.turns for x in tokens]
            sc = [x for _, scored in t.turns for x in scored]
            if not tk:
                raise ValueError(f"trajectory {t.tid} has no turns")
            toks.append(tk)
            masks.append(sc)
        groups = [self._groups[t.gid] for t in trajs]
        chains = [g.chain for g in groups]
        offs = [0] * len(trajs)
        hs: list[list[torch.Tensor]] = [[] for _ in trajs]
        blocked = False
        while True:
            live = [i for i in range(len(trajs)) if offs[i] < len(toks[i])]
            if not live:
                break
            ids, pos, segs = [], [], []
            cur = 0
            for i in live:
                n = len(toks[i]) - offs[i]
                if block is not None and n > block:
                    n = block
                    blocked = True
                ids.extend(toks[i][offs[i] : offs[i] + n])
                pos.append(self._positions(groups[i].prompt_len + offs[i], n))
                segs.append(Segment(cur, n, chains[i]))
                cur += n
            h, states = self._run_pack(self._ids(ids), torch.cat(pos), segs)
            for i, seg, st in zip(live, segs, states):
                hs[i].append(h[seg.start : seg.start + seg.length])
                chains[i] = self._chain_extend(chains[i], st)
                offs[i] += seg.length
        if rung in ("plain", "blocked"):
            rung = "blocked" if blocked else "plain"
        self._counts[rung] += 1
        self._last_rung = rung
        out = []
        for i, t in enumerate(trajs):
            h_all = hs[i][0] if len(hs[i]) == 1 else torch.cat(hs[i], 0)
            lp = self._scored_logprobs(h_all, groups[i].last, toks[i], masks[i])
            t.rebuilt = lp
            t.rebuilt_old = lp.detach()
            out.append(lp)
        return out

    # ------------------------------------------------------------ backward
    @contextlib.contextmanager
    def capture_source(self, source: Any):
        prev = self._capture_source
        self._capture_source = source
        try:
            yield
        finally:
            self._capture_source = prev

    def backward_with_boundary_adjoint_capture(
        self,
        tensors,
        grad_tensors=None,
        *,
        source: Any = None,
        retain_graph: bool = False,
        sink: GradSink | None = None,
    ) -> None:
        """Backward whose boundary-proxy gradients land in the fp32 ledgers."""
        with self.capture_source(source), grad_sink(sink):
            torch.autograd.backward(tensors, grad_tensors, retain_graph=retain_graph)

    def consume_boundary_adjoint_pairs(self, group_id: int):
        return self.boundary(group_id).consume()

    def drain_shared_prefix_source(self, group_id: int) -> list[torch.Tensor | None]:
        return self.boundary(group_id).drain()

    def finalize_group_boundary(
        self,
        group_id: int,
        adjoints: list[torch.Tensor | None] | None = None,
        *,
        sink: GradSink | None = None,
    ) -> None:
        """The one prompt backward of a group, with the summed (or given) adjoint."""
        g = self._groups[group_id]
        if g.boundary is None:
            return
        if adjoints is None:
            pairs = g.boundary.consume()
        else:
            if len(adjoints) != len(g.boundary.real):
                raise ValueError("one adjoint per boundary tensor")
            pairs = [(r, a.to(r.dtype)) for r, a in zip(g.boundary.real, adjoints) if a is not None]
            g.boundary._consumed = True
        pairs = [(r, a) for r, a in pairs if r.requires_grad]
        if pairs:
            with self.capture_source(("group_boundary", group_id)), grad_sink(sink):
                torch.autograd.backward([r for r, _ in pairs], [a for _, a in pairs])
        g.boundary.release()
        g.boundary = None
        g.real_graph = []
        if self.dependency_ready_shared_prefix_vjp and self.boundary_cut:
            self._dependency_ready_vjps(list(g.shared_nodes), sink)

    def finalize_trajectories_turn_boundaries(self, traj_ids: list[int], *, sink: GradSink | None = None) -> None:
        """Replay a closure cohort's cut turns last to first, carrying later turns' adjoints back (reference
        behaviour: src/thundersync/engine/streaming.py:6241-6330). Each round takes the latest unreplayed
        turn of every member; those the turn memory rule admits together (:meth:`_turn_replay_pack`) run
        as one joint pack with one backward, the rest wait for a later round."""
        members = [self._trajs[t] for t in traj_ids if t in self._trajs]
        while True:
            ready = []
            for t in members:
                while t.cuts and not t.cuts[-1].boundary.has_adjoint():
                    t.cuts.pop().boundary.release()
                if t.cuts:
                    ready.append(t)
            if not ready:
                return
            pick = self._turn_replay_pack([(len(t.cuts[-1].tokens), t.cuts[-1].pos0) for t in ready])
            batch = [ready[i] for i in pick]
            cuts = [t.cuts.pop() for t in batch]
            self._check_versions()
            ids: list[int] = []
            pos, segs, cur = [], [], 0
            for c in cuts:
                ids.extend(c.tokens)
                pos.append(self._positions(c.pos0, len(c.tokens)))
                segs.append(Segment(cur, len(c.tokens), c.parent_chain))
                cur += len(c.tokens)
            h, states = self._run_pack(self._ids(ids), torch.cat(pos), segs)
            reals, adjs = [], []
            for c, seg, st in zip(cuts, segs, states):
                real = _flatten_state(st, self.spec.kinds) + [h[seg.start + seg.length - 1]]
                for r, a in zip(real, c.boundary.peek()):
                    if a is not None:
                        reals.append(r)
                        adjs.append(a.to(r.dtype))
            self._counts["turn_replay"] += len(cuts)
            key = str(len(cuts))
            self._turn_counts["replay"][key] = self._turn_counts["replay"].get(key, 0) + 1
            if reals:
                src = ("turn_replay", batch[0].tid if len(batch) == 1 else tuple(t.tid for t in batch))
                with self.capture_source(src), grad_sink(sink):
                    torch.autograd.backward(reals, adjs)
            for c in cuts:
                c.boundary.release()

    def _shared_node_ready(self, node: _SharedNode) -> bool:
        """Every group under the node has run its prompt backward and every shared child is done."""
        if node.finalized:
            return False
        if any(not self._shared[c].finalized for c in node.children):
            return False
        return all(self._groups.get(gid) is None or self._groups[gid].boundary is None for gid in node.groups)

    def _run_shared_vjps(self, nodes: list[_SharedNode], sink: GradSink | None) -> None:
        """One autograd call over independent nodes (none is an ancestor of another; children are done)."""
        outs, grads = [], []
        for node in nodes:
            if node.boundary is not None:
                for r, a in node.boundary.consume():
                    if r.requires_grad:
                        outs.append(r)
                        grads.append(a)
        if outs:
            src = ("shared_prefix", nodes[0].idx) if len(nodes) == 1 else (
                "shared_prefix_frontier", tuple(n.idx for n in nodes))
            t0 = time.perf_counter() if self.shared_prefix_vjp_timing else 0.0
            with self.capture_source(src), grad_sink(sink):
                torch.autograd.backward(outs, grads)
            if self.shared_prefix_vjp_timing:
                if self.device.type == "cuda":
                    torch.cuda.synchronize(self.device)
                self._shared_prefix_times.append(time.perf_counter() - t0)
        for node in nodes:
            if node.boundary is not None:
                node.boundary.release()
                node.boundary = None
            node.finalized = True
            node.chain = None
        self._shared_prefix_calls += 1

    def _dependency_ready_vjps(self, start: list[int], sink: GradSink | None) -> None:
        """After a group's prompt backward: run each ancestor shared node, deepest first, once it is ready."""
        for idx in start:
            node = self._shared[idx]
            if not self._shared_node_ready(node):
                break
            self._run_shared_vjps([node], sink)
            self._shared_prefix_early += 1

    def finalize_shared_prefixes(self, *, sink: GradSink | None = None) -> int:
        """Backward every remaining shared prompt node once, children before parents: one autograd call
        per node (``shared_prefix_vjp_backend="sequential"``) or per frontier of nodes whose children are
        all done (``"ready_frontier"``)."""
        done = 0
        while True:
            pending = [n for n in reversed(self._shared) if not n.finalized]
            if not pending:
                return done
            frontier = [n for n in pending if all(self._shared[c].finalized for c in n.children)]
            if not frontier:
                raise RuntimeError("shared prompt forest has no node whose children are all done")
            batch = frontier if self.shared_prefix_vjp_backend == "ready_frontier" else frontier[:1]
            self._run_shared_vjps(batch, sink)
            done += len(batch)

    # ------------------------------------------------------------ parameter adjoints
    def accumulate_parameter_adjoint(self, parameter: torch.Tensor, value: torch.Tensor, *, source: Any = None) -> None:
        self.accumulate_parameter_adjoints([(parameter, value)], source=source)

    def accumulate_parameter_adjoints(self, pairs, *, source: Any = None) -> None:
        if self.parameter_adjoint_reduction == "canonical_source":
            dev = self._param_adjoint_device
            self._param_adjoint_staged.setdefault(source, []).extend(
                (p, v.detach().float().clone() if dev is None else v.detach().float().to(dev, copy=True))
                for p, v in pairs
            )
            return
        with torch.no_grad():
            for p, v in pairs:
                if p.grad is None:
                    p.grad = v.detach().to(p.dtype).clone()
                else:
                    p.grad.add_(v.to(p.grad.dtype))

    def materialize_parameter_adjoints(self) -> None:
        """Apply staged contributions in canonical (sorted source) order."""
        if not self._param_adjoint_staged:
            return
        acc: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}
        for src in sorted(self._param_adjoint_staged, key=repr):
            for p, v in self._param_adjoint_staged[src]:
                if id(p) in acc:
                    acc[id(p)][1].add_(v)
                else:
                    acc[id(p)] = (p, v)
        with torch.no_grad():
            for p, v in acc.values():
                if p.grad is None:
                    p.grad = v.to(device=p.device, dtype=p.dtype)
                else:
                    p.grad.add_(v.to(device=p.grad.device, dtype=p.grad.dtype))
        self._param_adjoint_staged.clear()

    # ------------------------------------------------------------ lifecycle
    def free_trajectory(self, traj_id: int) -> None:
        t = self._trajs.pop(traj_id, None)
        if t is None:
            return
        for c in t.cuts:
            c.boundary.release()
        t.cuts.clear()
        t.chain = []
        t.logprobs.clear()
        t.old.clear()
        t.rebuilt = None
        t.rebuilt_old = None

    def free_group(self, group_id: int) -> None:
        g = self._groups.get(group_id)
        if g is None:
            return
        for tid in list(g.trajs):
            self.free_trajectory(tid)
        if g.boundary is not None:
            g.boundary.release()
            g.boundary = None
        g.chain = []
        g.real_graph = []
        g.closed = True

    def close(self) -> None:
        for gid in list(self._groups):
            self.free_group(gid)
        for node in self._shared:
            if node.boundary is not None:
                node.boundary.release()
        self._shared.clear()
        if self in _LIVE:
            _LIVE.remove(self)

    # ------------------------------------------------------------ diagnostics
    def kv_bytes_resident(self) -> int:
        seen: set[int] = set()
        total = 0
        chains = [g.chain for g in self._groups.values()] + [t.chain for t in self._trajs.values()]
        for chain in chains:
            for t in _flatten_chain(chain):
                key = t.data_ptr()
                if key not in seen:
                    seen.add(key)
                    total += t.numel() * t.element_size()
        return total

    def retained_device_bytes(self) -> dict[str, int]:
        out = {"kv": self.kv_bytes_resident(), "ledgers": 0, "logprobs": 0}
        for g in self._groups.values():
            if g.boundary is not None:
                out["ledgers"] += sum(x.numel() * x.element_size() for x in g.boundary.peek() if x is not None)
        for t in self._trajs.values():
            out["logprobs"] += sum(x.numel() * x.element_size() for x in t.logprobs)
        out["total"] = sum(out.values())
        return out

    def prompt_token_accounting(self) -> dict[str, Any]:
        h = hashlib.sha256()
        for gid in sorted(self._groups):
            h.update(str((gid, self._groups[gid].prompt_len, self._groups[gid].shared_nodes)).encode())
        return {
            "physical_prompt_tokens": self._prompt_tokens_physical,
            "logical_prompt_tokens": self._prompt_tokens_logical,
            "sharing": round(self._prompt_tokens_logical / max(self._prompt_tokens_physical, 1), 4),
            "shared_nodes": len(self._shared),
            "topology_sha256": h.hexdigest(),
        }

    @property
    def rebuild_path_counts(self) -> dict[str, int]:
        return {k: self._counts[k] for k in self.REBUILD_RUNGS} | {"oom_retries": self._oom_retries}

    @property
    def turn_path_counts(self) -> dict[str, dict[str, int]]:
        return {k: dict(v) for k, v in self._turn_counts.items()}

    @property
    def last_rebuild_rung(self) -> str | None:
        return self._last_rung

    def rebuild_checkpoint_storage_device(self):
        return self._rebuild_checkpoint_storage_device

    def rebuild_checkpoint_offload_diagnostics(self) -> dict[str, Any]:
        """Bytes the checkpoint rungs parked in host memory (written) and brought back (read)."""
        dev = self._rebuild_checkpoint_storage_device
        return {"device": None if dev is None else str(dev), "write_bytes": self._offload["write_bytes"],
                "read_bytes": self._offload["read_bytes"], "tensors": self._offload["tensors"],
                "host_rebuilds": self._counts["checkpoint_host"]}

    def parameter_adjoint_diagnostics(self) -> dict[str, Any]:
        return {
            "reduction": self.parameter_adjoint_reduction,
            "staged_sources": len(self._param_adjoint_staged),
            "storage_device": None if self._param_adjoint_device is None else str(self._param_adjoint_device),
            "staged_bytes": sum(v.numel() * v.element_size() for st in self._param_adjoint_staged.values()
                                for _, v in st),
        }

    def shared_prefix_vjp_diagnostics(self) -> dict[str, Any]:
        out = {
            "backend": self.shared_prefix_vjp_backend,
            "nodes": len(self._shared),
            "finalized": sum(1 for n in self._shared if n.finalized),
            "autograd_calls": self._shared_prefix_calls,
            "dependency_ready": self.dependency_ready_shared_prefix_vjp,
            "finalized_before_barrier": self._shared_prefix_early,
        }
        if self.shared_prefix_vjp_timing:  # wall seconds per shared-prefix backward (device-synchronised)
            out["vjp_seconds"] = list(self._shared_prefix_times)
            out["vjp_seconds_total"] = float(sum(self._shared_prefix_times))
        return out

    def shared_prefix_finalization_diagnostics(self) -> dict[str, Any]:
        """The shared-prefix VJP state under the reference's older name (same record as
        :meth:`shared_prefix_vjp_diagnostics`)."""
        return self.shared_prefix_vjp_diagnostics()

    def close_memory_window(self) -> None:
        """Record the open window's measured peak above its start (allocator counters, no device sync)."""
        w = self._memory_window
        if w is None:
            return
        self._memory_window = None
        peak = int(torch.cuda.max_memory_allocated(self.device))
        w["measured"] = max(0, peak - w["allocated"])
        self._memory_windows.append(w)

    @property
    def turn_memory_windows(self) -> list[dict[str, Any]]:
        """Every closed memory window of this run (phase, executor, estimate, measured), in call order."""
        self.close_memory_window()
        return list(self._memory_windows)

    @property
    def turn_memory_report(self) -> dict[str, Any]:
        """The memory rule's estimates against measured peaks, per phase/executor, and its refusals.

        ``windows[phase/executor]``: calls, the largest estimate and measured peak above the call's start,
        the largest measured/estimate ratio and how many calls exceeded their estimate. ``refused`` counts
        rungs the rule turned down for lack of memory; ``allocator_retries`` counts allocations that had
        to free cached blocks first since the first window.
        """
        self.close_memory_window()
        out: dict[str, dict[str, Any]] = {}
        for w in self._memory_windows:
            r = out.setdefault(f"{w['phase']}/{w['executor']}", {"calls": 0, "max_estimate_bytes": 0,
                                                                  "max_measured_bytes": 0,
                                                                  "max_measured_over_estimate": 0.0, "exceeded": 0})
            r["calls"] += 1
            r["max_estimate_bytes"] = max(r["max_estimate_bytes"], w["estimate"])
            r["max_measured_bytes"] = max(r["max_measured_bytes"], w["measured"])
            if w["estimate"]:
                r["max_measured_over_estimate"] = max(r["max_measured_over_estimate"],
                                                      round(w["measured"] / w["estimate"], 4))
            r["exceeded"] += int(w["measured"] > w["estimate"])
        retries = None
        if self._memory_retries_at_start is not None:
            retries = int(torch.cuda.memory_stats(self.device).get("num_alloc_retries", 0)) - \
                self._memory_retries_at_start
        return {"reserve_bytes": self.rebuild_plain_reserve_bytes, "activation_factor": TURN_ACTIVATION_FACTOR,
                "refused": dict(sorted(self._memory_refusals.items())),
                "min_available_bytes": self._memory_min_available, "allocator_retries": retries,
                "oom_retries": self._oom_retries, "windows": out}


def _flatten_chain(chain: list[Any]) -> list[torch.Tensor]:
    out: list[torch.Tensor] = []
    for st in chain:
        if st is None:
            continue
        for part in st:
            if isinstance(part, list):
                out.extend(part)
            elif isinstance(part, torch.Tensor):
                out.append(part)
    return out


def _unflatten_chain(chain: list[Any], flat: list[torch.Tensor]) -> list[Any]:
    it = iter(flat)
    out = []
    for st in chain:
        if st is None:
            out.append(None)
            continue
        parts = []
        for part in st:
            if isinstance(part, list):
                parts.append([next(it) for _ in part])
            elif isinstance(part, torch.Tensor):
                parts.append(next(it))
            else:
                parts.append(part)
        out.append(tuple(parts))
    return out


def _own_only(states: list[Any]) -> list[Any]:
    return states
