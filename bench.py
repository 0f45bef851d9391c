"""Streaming-GRPO throughput benchmark (default: config 2, Qwen3-1.7B full fine-tune).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2|3|5]

``--config 3``: Qwen3-8B architecture with LoRA r64/alpha 128 on q/k/v/o/gate/up/down (frozen bf16 base,
fp32 adapters), agentic multi-turn GRPO: per rank 4 groups x 16 trajectories (32 x 16 at 8 GPUs), a
2048-token prompt, 4-16 turns of U[128,1024] scored action tokens followed by U[64,2048] unscored tool
tokens, context capped at 32768, rewards U[0,1].
``--config 5``: hybrid 48-layer model (3x gated DeltaNet + 1x gated attention, GQA 16/2, head_dim 256),
per rank 2 groups x 8 trajectories (16 x 8 at 8 GPUs), 1024-token prompt, completions U[4096,32768],
rewards Bernoulli(0.5).

For N > 1 launch one process per GPU with torch.distributed.run; every rank
reads RANK / LOCAL_RANK / WORLD_SIZE / MASTER_* from the environment.

Workload per rank and step (weak scaling: fixed per GPU, 64 groups total at 8
GPUs): 8 groups x 8 trajectories of a random-init Qwen3-1.7B-architecture
model in bf16 (fp32 master weights and Adam moments). Prompts are 512 uniform
token ids, completions uniform in [256, 4096] tokens, every completion token
scored, rewards Bernoulli(0.3). Each trajectory's completion time is
Exponential(mean 2 s); trajectories are delivered in that arrival order, as
fast as the trainer consumes them, so groups interleave exactly as they
would under streaming arrival.

One step = open every group (prompt forward), then for each arrival:
append_turn + close_trajectory (reward arrives; the trajectory is
differentiated and folded), close_group when a group's last reward lands,
then the DP step (gradient mean across ranks, clip 1.0, AdamW maximize).

Reported: scored completion tokens per second for the whole job (device-timed
with CUDA events around K steps, max over ranks), and the post-last-reward
tail: device time from the delivery of the step's last reward to the end of
the optimizer step. The e2e figure is wall-clock over the same steps through
the public API, which copies each step's token ids host->device from pinned
memory and reads the gradient norm back.
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import random
import statistics
import subprocess
import sys
import tempfile
import time
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "scored tokens/sec/box per GRPO step"
BASELINE_VALUE = None  # the reference publishes no number for this metric


# ----------------------------------------------------------------------------- workload
CONFIGS = {
    2: dict(model="qwen3-1.7b", groups_per_rank=8, group_size=8, prompt_len=512, min_len=256, max_len=4096,
            rewards="bernoulli", reward_p=0.3, lora=0),
    3: dict(model="qwen3-8b", groups_per_rank=4, group_size=16, prompt_len=2048, rewards="uniform", lora=64,
            lora_alpha=128, turns=(4, 16), scored=(128, 1024), unscored=(64, 2048), context_cap=32768),
    4: dict(model="qwen3-4b", groups_per_rank=32, group_size=1, prompt_len=512, rewards="teacher", lora=0,
            actions=(8, 32), action_tokens=(64, 512), observation_tokens=(32, 512), teacher_mean=1.5,
            teacher_latency_s=0.5),
    5: dict(model="hybrid-48l", groups_per_rank=2, group_size=8, prompt_len=1024, min_len=4096, max_len=32768,
            rewards="bernoulli", reward_p=0.5, lora=0),
}


def make_step_opd(rank: int, step: int, args) -> dict:
    """Config 4: per rank 32 single-trajectory groups (256 at 8 GPUs), each 8-32 actions of U[64,512] scored
    tokens after U[32,512] unscored observation tokens; teacher log-probs -Exp(mean 1.5) clipped to [-20, 0]
    arrive per action after Exp(mean 0.5 s); actions are delivered in that arrival order."""
    c = CONFIGS[4]
    rng = random.Random(args.seed * 1_000_003 + rank * 10_007 + step)
    groups, events = [], []
    for g in range(args.groups_per_rank):
        prompt = [rng.randrange(args.vocab) for _ in range(args.prompt_len)]
        groups.append((g, prompt, [g]))
        t = 0.0
        n_act = rng.randint(*c["actions"])
        for k in range(n_act):
            obs = [rng.randrange(args.vocab) for _ in range(rng.randint(*c["observation_tokens"]))] if k else []
            act = [rng.randrange(args.vocab) for _ in range(rng.randint(*c["action_tokens"]))]
            teacher = [max(-20.0, -rng.expovariate(1.0 / c["teacher_mean"])) for _ in act]
            t += rng.expovariate(1.0 / c["teacher_latency_s"])
            events.append((t, g, k, obs + act, [False] * len(obs) + [True] * len(act), teacher, k == n_act - 1))
    events.sort(key=lambda e: e[0])
    scored = sum(sum(e[4]) for e in events)
    tokens = sum(len(e[3]) for e in events) + sum(len(p) for _, p, _ in groups)
    return {"groups": groups, "events": events, "scored": scored, "tokens": tokens}


def opd_open_budget(args, device) -> int:
    """How many config-4 trajectories fit on the device at once: the memory left beside the model (bf16
    weights, fp32 master / Adam moments / gradient) over an open trajectory's retained bytes at 1.5x the
    expected length (its K/V in bf16 plus fp32 adjoint ledgers of the same rows: 3x the K/V bytes)."""
    from thundersync_b200.models.qwen3 import PRESETS

    cfg = PRESETS[args.model]
    c = CONFIGS[4]
    n_params = sum(p.numel() for p in _param_shapes(cfg))
    static = n_params * (2 + 4 + 4 + 4 + 4)
    head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
    kv_token = 2 * cfg.num_key_value_heads * head_dim * 2 * cfg.num_hidden_layers
    mean_actions = sum(c["actions"]) / 2
    mean_tokens = args.prompt_len + mean_actions * (sum(c["action_tokens"]) / 2 + sum(c["observation_tokens"]) / 2)
    total = torch.cuda.get_device_properties(device).total_memory
    # a joint pack's activations (about 16 hidden-width bf16 rows per token and layer, up to 4096 tokens)
    # plus 8 GB for workspaces
    pack_act = 4096 * cfg.num_hidden_layers * cfg.hidden_size * 2 * 16
    room = 0.85 * (total - static) - pack_act - (8 << 30)
    return max(1, int(room // (1.5 * mean_tokens * 3 * kv_token)))


def _param_shapes(cfg):
    """Parameter tensors of the Qwen3 architecture ``cfg`` (meta device: shapes only)."""
    from thundersync_b200.models.qwen3 import Qwen3ForCausalLM

    with torch.device("meta"):
        return list(Qwen3ForCausalLM(cfg).parameters())


class OPDTrainer:
    """Config 4 driver over either package's public OPD API: a run and an ``OPDTurnStream`` per batch, the
    step's gradient (normalised by the batch's scored-token count across ranks) and the optimizer."""

    def __init__(self, model, make_run, make_objective, optimizer, device, world, flat=None, reducer=None):
        self.model, self.make_run, self.make_objective = model, make_run, make_objective
        self.opt, self.device, self.world = optimizer, device, world
        self.flat, self.reducer = flat, reducer
        self.open_budget = None  # most trajectories streaming at once (None: all of the batch's)
        self.pack_limit = 16  # most actions in one joint scored-turn pack
        self.pack_tokens = 4096  # most tokens in one joint pack (its activations live until its backward)
        self.packs = self.packed_actions = 0
        self._new()

    def _new(self):
        self.run = self.make_run(self.model)
        self.obj = self.make_objective(self.run, self.model)
        if self.reducer is not None:
            self.obj.use_main_grad_buffer(self.reducer.main_grad_buffer())

    def step_batch(self, work, tail_start=None) -> dict:
        """Deliver the actions as they arrive. The step keeps a clock: each event's arrival time is its
        teacher score's latency after the step starts; the clock advances by the host time the trainer spends
        on each call (idle time before an arrival is skipped, not counted). Everything that has arrived by
        the clock and is not yet delivered is *ready*; each call hands the ready actions of distinct
        trajectories (a trajectory's actions in order) to the objective as one joint scored-turn pack, up to
        ``pack_limit`` actions and ``pack_tokens`` tokens. With ``open_budget`` at most that many trajectories stream at once (each
        open trajectory keeps its K/V and its turn boundaries' fp32 adjoint ledgers on the device until it
        closes); the others' actions stay ready until one closes. Same driver for both arms."""
        events = list(work["events"])
        n = len(events)
        prompts = {g: prompt for g, prompt, _ in work["groups"]}
        budget = self.open_budget
        opened: set = set()
        ready: list = []
        nxt, done, clock = 0, 0, 0.0
        while done < n:
            while nxt < n and events[nxt][0] <= clock:
                ready.append(events[nxt])
                nxt += 1
            if not ready:
                clock = events[nxt][0]
                continue
            pack, taken, blocked = [], set(), set()
            for ev in ready:
                g = ev[1]
                if g in taken or g in blocked:
                    blocked.add(g)  # this trajectory's later actions wait for the earlier one
                    continue
                if g not in opened and budget is not None and len(opened) + len(
                        [x for x in taken if x not in opened]) >= budget:
                    blocked.add(g)
                    continue
                if pack and sum(len(e[3]) for e in pack) + len(ev[3]) > self.pack_tokens:
                    break
                pack.append(ev)
                taken.add(g)
                if len(pack) >= self.pack_limit:
                    break
            if not pack:  # every ready action waits for a slot: the open trajectories' next actions come later
                if nxt >= n:
                    raise RuntimeError("open-trajectory budget admits nothing")
                clock = max(clock, events[nxt][0])
                continue
            t0 = time.perf_counter()
            for ev in pack:
                ready.remove(ev)
                if ev[1] not in opened:
                    opened.add(ev[1])
                    self.obj.open_group(ev[1], prompts[ev[1]])
            done += len(pack)
            if done == n and tail_start is not None:
                tail_start.record()  # the step's last teacher score reaches the trainer: the tail starts
            items = [(g, g, toks, mask, torch.tensor(teacher, dtype=torch.float32).to(self.device, non_blocking=True),
                      None) for _, g, _, toks, mask, teacher, _ in pack]
            self.obj.append_scored_turns(items, return_loss=False)
            closing = [ev[1] for ev in pack if ev[6]]
            if closing:
                self.obj.close_trajectories(closing)
                for g in closing:
                    self.obj.close_group(g)
                    opened.discard(g)
            self.packs += 1
            self.packed_actions += len(pack)
            clock += time.perf_counter() - t0
        return self.finish()

    def finish(self) -> dict:
        if self.flat:
            self.obj.assert_safe_to_step(materialize=False)
            grad = self.obj.main_grad()
            if self.world > 1:
                # the objective divided by its local scored-token mass; the step wants the global mass
                mass = torch.tensor([self.obj.normalization_divisor], dtype=torch.float64, device=self.device)
                dist.all_reduce(mass)
                scale = self.world * self.obj.normalization_divisor / float(mass)
                self.reducer.all_reduce_mean(grad, pre_scale=scale)
            from thundersync_b200.parallel.optimizer import global_sq_norm

            coef, nrm = self.opt.clip_coefficient(global_sq_norm(grad), 1.0)
            self.opt.step(grad, clip_coef=coef)
        else:
            self.obj.assert_safe_to_step()
            params = [p for p in self.model.parameters() if p.requires_grad]
            if self.world > 1:
                for p in params:
                    dist.all_reduce(p.grad)
                    p.grad.div_(self.world)
            nrm = torch.nn.utils.clip_grad_norm_(params, 1.0)
            self.opt.step()
            self.opt.zero_grad(set_to_none=True)
        self.run.close() if hasattr(self.run, "close") else None
        self._new()
        return {"global_grad_norm": float(nrm)}


def _turns(rng: random.Random, args) -> list[tuple[list[int], list[bool]]]:
    """One trajectory's turns: one scored completion (configs 2, 5) or agentic (scored action, unscored
    tool output) turns within the context cap (config 3)."""
    c = CONFIGS[args.config]
    if "turns" not in c:
        n = rng.randint(args.min_len, args.max_len)
        return [([rng.randrange(args.vocab) for _ in range(n)], [True] * n)]
    room = c["context_cap"] - args.prompt_len
    out = []
    for _ in range(rng.randint(*c["turns"])):
        a = rng.randint(*c["scored"])
        o = rng.randint(*c["unscored"])
        if a + o > room:
            a = min(a, room)
            o = max(0, min(o, room - a))
        if a <= 0:
            break
        toks = [rng.randrange(args.vocab) for _ in range(a + o)]
        out.append((toks, [True] * a + [False] * o))
        room -= a + o
    return out


def make_step(rank: int, step: int, args) -> dict:
    rng = random.Random(args.seed * 1_000_003 + rank * 10_007 + step)
    groups = []
    arrivals = []
    for g in range(args.groups_per_rank):
        prompt = [rng.randrange(args.vocab) for _ in range(args.prompt_len)]
        tids = []
        for j in range(args.group_size):
            tid = g * args.group_size + j
            turns = _turns(rng, args)
            if CONFIGS[args.config]["rewards"] == "uniform":
                reward = rng.random()
            else:
                reward = 1.0 if rng.random() < args.reward_p else 0.0
            t_arrive = rng.expovariate(1.0 / args.mean_arrival_s)
            arrivals.append((t_arrive, g, tid, turns, reward))
            tids.append(tid)
        groups.append((g, prompt, tids))
    arrivals.sort(key=lambda a: a[0])
    scored = sum(sum(m) for a in arrivals for _, mask in a[3] for m in [mask])
    tokens = sum(len(t) for a in arrivals for t, _ in a[3]) + sum(len(p) for _, p, _ in groups)
    return {"groups": groups, "arrivals": arrivals, "scored": scored, "tokens": tokens}


def run_step(trainer, work, tail_start: torch.cuda.Event | None):
    if isinstance(trainer, OPDTrainer):
        return trainer.step_batch(work, tail_start)
    remaining = {g: len(tids) for g, _, tids in work["groups"]}
    for g, prompt, tids in work["groups"]:
        trainer.open_group(g, prompt)
        trainer.register_group_trajectories(g, tids)
    n = len(work["arrivals"])
    for i, (_, g, tid, turns, reward) in enumerate(work["arrivals"]):
        for tokens, mask in turns:
            trainer.append_turn(g, tid, tokens, mask)
        if i == n - 1 and tail_start is not None:
            tail_start.record()
        trainer.close_trajectory(tid, reward)
        remaining[g] -= 1
        if remaining[g] == 0:
            trainer.close_group(g)
    return trainer.step()


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, path: str) -> None:
        self.path = path
        self.proc = None

    def start(self) -> None:
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self, gpu_indices: list[int]) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        visible = os.environ.get("CUDA_VISIBLE_DEVICES")
        phys = [int(x) for x in visible.split(",")] if visible else gpu_indices
        want = {phys[i] if i < len(phys) else i for i in gpu_indices}
        with open(self.path) as fh:
            for line in fh:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    idx = int(parts[0])
                except ValueError:
                    continue
                if idx not in want:
                    continue
                try:
                    sm.append(float(parts[1]))
                    mx.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(names, parts[5:9]):
                    if val.lower() in ("active", "1", "yes"):
                        reasons.add(name)
        busy = [s for s in sm if s > 0.5 * (max(mx) if mx else 1)] or sm
        return {
            "sm_mhz": statistics.median(busy) if busy else None,
            "sm_max_mhz": max(mx) if mx else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ----------------------------------------------------------------------------- arms
def build_ours(args, device):
    from thundersync_b200.grpo.data_parallel import DataParallelThunderSync
    from thundersync_b200.models.qwen3 import PRESETS, Qwen3ForCausalLM
    from thundersync_b200.engine.streaming import StreamingRun, arena_for
    from thundersync_b200.parallel.optimizer import FlatAdamW

    torch.manual_seed(args.seed)
    if args.model.startswith("hybrid"):
        from thundersync_b200.models.hybrid import HYBRID_PRESETS, HybridForCausalLM

        with torch.device(device):
            model = HybridForCausalLM(HYBRID_PRESETS[args.model])
    else:
        with torch.device(device):
            model = Qwen3ForCausalLM(PRESETS[args.model])
    model.to(dtype=torch.bfloat16)
    c = CONFIGS[args.config]
    if c["lora"]:
        from thundersync_b200.policy_model import apply_lora

        _, model = apply_lora(model, rank=c["lora"], alpha=c["lora_alpha"])
    arena = arena_for(model)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    # config 2: data parallel with a sharded optimizer (ZeRO-1: reduce-scatter -> shard AdamW -> bf16 gather)
    make = FlatAdamW.sharded if world > 1 else FlatAdamW
    opt = make(arena, lr=args.lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, maximize=True)

    def factory(m):
        return StreamingRun(m, boundary_cut=True, checkpoint=False, stream_turns=False,
                            rebuild_block_tokens=args.block_tokens)

    trainer = DataParallelThunderSync.init_from_env(
        model, opt, run_factory=factory, grad_clip=1.0,
        source_offload_device=None, source_offload_mode="device_resident",
    )
    if CONFIGS[args.config]["rewards"] == "bernoulli":
        trainer.configure_binary_rewards()
    return model, trainer


def _reference_snapshot(args, device, c) -> str:
    """Write a random-init Hugging Face snapshot of the benchmark model once per host.

    The reference's builder loads its policy from a snapshot directory
    (``load_policy_model`` -> ``from_pretrained``); there is no network, so the
    snapshot is the architecture's own random init (N(0, 0.02), seeded), saved
    in bf16. Local rank 0 writes it; the other ranks wait on the barrier, and the
    reference's ``init_from_env`` broadcasts rank 0's weights anyway.
    """
    from transformers import AutoConfig, AutoModelForCausalLM

    path = os.path.join(args.ref_snapshot_dir, f"{args.model}-seed{args.seed}")
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if local == 0 and not os.path.isfile(os.path.join(path, "config.json")):
        hf_cfg = AutoConfig.for_model(
            "qwen3", vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
            num_hidden_layers=c.num_hidden_layers, num_attention_heads=c.num_attention_heads,
            num_key_value_heads=c.num_key_value_heads, head_dim=c.head_dim, rms_norm_eps=c.rms_norm_eps,
            rope_theta=c.rope_theta, tie_word_embeddings=c.tie_word_embeddings,
            max_position_embeddings=c.max_position_embeddings, initializer_range=c.initializer_range,
        )
        torch.manual_seed(args.seed)
        with torch.device(device):
            model = AutoModelForCausalLM.from_config(hf_cfg, dtype=torch.bfloat16)
        tmp = path + f".tmp{os.getpid()}"
        model.save_pretrained(tmp)
        del model
        torch.cuda.empty_cache()
        os.replace(tmp, path)
    if dist.is_initialized():
        dist.barrier()
    return path


def build_ours_opd(args, device, world):
    from thundersync_b200.engine.streaming import StreamingRun, arena_for
    from thundersync_b200.models.qwen3 import PRESETS, Qwen3ForCausalLM
    from thundersync_b200.opd.objectives import OPDTurnStream
    from thundersync_b200.parallel.optimizer import FlatAdamW

    torch.manual_seed(args.seed)
    with torch.device(device):
        model = Qwen3ForCausalLM(PRESETS[args.model])
    model.to(dtype=torch.bfloat16).eval()  # turn replay needs a deterministic forward
    arena = arena_for(model)
    reducer = None
    if world > 1:
        from thundersync_b200.parallel.reduce import GradientReducer

        with torch.no_grad():
            dist.broadcast(arena.flat, src=0)
        reducer = GradientReducer(arena.numel, device, arena=arena)
    opt = FlatAdamW(arena, lr=args.lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0)
    return model, OPDTrainer(
        model, lambda m: StreamingRun(m, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True),
        lambda r, m: OPDTurnStream(r, m), opt, device, world, flat=True, reducer=reducer)


def build_reference_opd(args, device, world):
    """The reference's OPD objective through its public API (``StreamingRun`` + ``OPDTurnStream``, torch
    AdamW; reference src/thundersync/opd/objectives.py:947-1180) on the same random-init snapshot."""
    from thundersync import STREAM_ATTENTION_NAME, register_stream_attention
    from thundersync.engine.streaming import StreamingRun
    from thundersync.opd.objectives import OPDTurnStream
    from transformers import AutoModelForCausalLM

    from thundersync_b200.models.qwen3 import PRESETS

    snapshot = _reference_snapshot(args, device, PRESETS[args.model])
    register_stream_attention()
    model = AutoModelForCausalLM.from_pretrained(snapshot, dtype=torch.bfloat16,
                                                 attn_implementation=STREAM_ATTENTION_NAME,
                                                 local_files_only=True).to(device)
    model.config.use_cache = False
    model.eval()
    if world > 1:
        with torch.no_grad():
            for t in model.state_dict().values():
                dist.broadcast(t, src=0)
    opt = torch.optim.AdamW([p for p in model.parameters() if p.requires_grad], lr=args.lr, betas=(0.9, 0.999),
                            eps=1e-8, weight_decay=0.0)
    return model, OPDTrainer(
        model, lambda m: StreamingRun(m, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True),
        lambda r, m: OPDTurnStream(r, m), opt, device, world, flat=False)


def build_reference(args, device):
    """The unmodified reference, built by its own production builder.

    Path: ``GrpoTrainerConfig.from_namespace`` (the reference's entry-point
    translation) -> ``thundersync.grpo.runtime.load_trainer`` (reference
    ``src/thundersync/grpo/runtime.py:151-319``), which loads the policy from a
    snapshot, picks the source-attention backend after its own device trial,
    builds AdamW(maximize) or, at N > 1, its ZeRO-1 ``ShardedOptimizerStep``,
    places the group statistics (``statistic_device="auto"``) and returns its
    ``DataParallelThunderSync``. Nothing from this package runs on that path;
    only the model preset's numbers are read from here.
    """
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "thundersync")):
        raise RuntimeError("reference not installed under baseline/_ref")
    if args.config == 3:
        import importlib.util

        if importlib.util.find_spec("peft") is None:
            raise RuntimeError("config 3 needs the reference's LoRA path (thundersync.policy_model.apply_lora), "
                               "which imports peft; peft is not installed on this image")
    if args.config == 5:
        raise RuntimeError("config 5 runs the reference's hybrid layers through flash-linear-attention's "
                           "chunk_gated_delta_rule, which raised a misaligned-address fault on this pool's "
                           "B200s; it is not run again")
    sys.path.insert(0, ref)
    from types import SimpleNamespace

    from thundersync import register_stream_attention
    from thundersync.grpo.config import GrpoTrainerConfig
    from thundersync.grpo.runtime import load_trainer

    from thundersync_b200.models.qwen3 import PRESETS

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if not dist.is_initialized():
        os.environ.setdefault("RANK", "0")
        os.environ.setdefault("WORLD_SIZE", "1")
        os.environ.setdefault("LOCAL_RANK", "0")
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", str(29500 + os.getpid() % 1000))
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=900))
    snapshot = _reference_snapshot(args, device, PRESETS[args.model])
    if args.ref_deterministic:
        os.environ.setdefault("CUBLAS_WORKSPACE_CONFIG", ":4096:8")
    ns = SimpleNamespace(
        model_path=snapshot,
        learning_rate=args.lr,
        rebuild_block_tokens=args.block_tokens,
        grad_clip=1.0,
        optimizer_state_sharding=world > 1,
        deterministic_algorithms=bool(args.ref_deterministic),
        compile_pointwise_modules=bool(args.ref_compile),
        source_offload_device="cpu",
        source_offload_mode="device_resident",
        statistic_device="auto",
        statistic_open_groups=args.groups_per_rank,
        source_attention_backend=args.ref_attention,
    )
    config = GrpoTrainerConfig.from_namespace(ns)
    # the builder's "auto" backend names the stream attention, which the
    # reference's entry points register with transformers first
    register_stream_attention()
    model, _optimizer, trainer = load_trainer(config, device)
    trainer.configure_binary_rewards()
    return model, trainer


def reference_diagnostics() -> dict:
    """Which attention paths and kernel trials the reference's run used."""
    from thundersync.accel.capability import kernel_probe_records
    from thundersync.engine.streaming import attention_path_counts

    probes = []
    for rec in kernel_probe_records():
        probes.append({k: rec.get(k) for k in ("kernel", "runs", "error") if k in rec})
    return {"attention_path_counts": attention_path_counts(), "kernel_probes": probes}


# ----------------------------------------------------------------------------- main
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS),
                    help="BASELINE workload: 2 (Qwen3-1.7B full FT), 3 (Qwen3-8B LoRA agentic), 5 (hybrid)")
    ap.add_argument("--model", default=None)
    ap.add_argument("--groups-per-rank", type=int, default=None)
    ap.add_argument("--group-size", type=int, default=None)
    ap.add_argument("--prompt-len", type=int, default=None)
    ap.add_argument("--min-len", type=int, default=None)
    ap.add_argument("--max-len", type=int, default=None)
    ap.add_argument("--reward-p", type=float, default=None)
    ap.add_argument("--mean-arrival-s", type=float, default=2.0)
    ap.add_argument("--block-tokens", type=int, default=4096)
    ap.add_argument("--opd-open-trajectories", type=int, default=0,
                    help="config 4: most trajectories streaming at once per rank (0: from the device memory)")
    ap.add_argument("--lr", type=float, default=1e-5)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--clocks-file", default=None,
                    help="where nvidia-smi clock samples of the timed region are written (default: a temp file)")
    ap.add_argument("--ref-attention", default="cudnn_graph", choices=["auto", "cudnn", "cudnn_graph"],
                    help="reference arm: source_attention_backend given to its builder (cudnn_graph, its fastest "
                         "measured on B200, if its device trial passes)")
    ap.add_argument("--ref-compile", type=int, default=0,
                    help="reference arm: compile_pointwise_modules (torch.compile of MLP and norms)")
    ap.add_argument("--ref-deterministic", type=int, default=0,
                    help="reference arm: deterministic_algorithms")
    ap.add_argument("--ref-snapshot-dir", default=os.path.join(tempfile.gettempdir(), "thundersync_ref_snapshots"),
                    help="reference arm: where the random-init snapshot its builder loads is written")
    ap.add_argument("--profile-out", default=None,
                    help="after the timed region, run one more step under torch.profiler and write the per-kernel "
                         "CUDA time table to this file (rank 0; not part of any reported number)")
    ap.add_argument("--cprofile-out", default=None,
                    help="after the timed region, run one more step under cProfile and write the host-side "
                         "function table (by own time) to this file (rank 0; not part of any reported number)")
    args = ap.parse_args()
    for key, value in CONFIGS[args.config].items():  # the config's shape unless a flag overrides it
        if key in ("model", "groups_per_rank", "group_size", "prompt_len", "min_len", "max_len", "reward_p") \
                and getattr(args, key) is None:
            setattr(args, key, value)
    if args.warmup < 3:
        raise SystemExit("at least 3 warm-up steps are required")
    if args.config == 4:
        # open trajectories of unequal lengths free and allocate blocks of every size; expandable segments keep
        # the freed space usable (set before the first CUDA allocation; both arms)
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=900))

    c = CONFIGS[args.config]
    if c["lora"]:
        model_desc = (f"{args.model} architecture, random init N(0,0.02), frozen bf16 base, LoRA r{c['lora']} "
                      f"alpha {c['lora_alpha']} on q/k/v/o/gate/up/down (fp32 adapters, fp32 Adam)")
        seq = (f"prompt {args.prompt_len} + {c['turns'][0]}-{c['turns'][1]} turns of U{list(c['scored'])} scored "
               f"+ U{list(c['unscored'])} unscored tokens, context cap {c['context_cap']}")
    else:
        model_desc = f"{args.model} architecture, random init N(0,0.02), bf16 weights, fp32 master/Adam"
        seq = f"prompt {args.prompt_len} + completion U[{args.min_len},{args.max_len}]"
    if args.config == 4:
        model_desc = f"{args.model} architecture (OPD student), random init N(0,0.02), bf16 weights, fp32 master/Adam"
        seq = (f"prompt {args.prompt_len} + {c['actions'][0]}-{c['actions'][1]} actions of U{list(c['action_tokens'])} "
               f"scored tokens after U{list(c['observation_tokens'])} unscored observation tokens")
    rewards = ("U[0,1]" if c["rewards"] == "uniform" else
               "teacher log-probs -Exp(mean 1.5) clipped to [-20,0], per action after Exp(mean 0.5 s)"
               if c["rewards"] == "teacher" else f"Bernoulli({args.reward_p})")
    cfg_block = {
        "baseline_config": args.config,
        "model": model_desc,
        "global_batch": (f"{args.groups_per_rank * world} trajectories" if args.config == 4 else
                         f"{args.groups_per_rank * world} groups x {args.group_size} trajectories"),
        "seq_len": seq,
        "parallelism": f"dp{world}",
        "rewards": rewards if args.config == 4 else f"{rewards}, arrival order Exp(mean {args.mean_arrival_s}s)",
        "l2": "no flush needed: every step streams > 3 GB of weights and GBs of statistics (L2 126 MB)",
    }
    try:
        if args.config == 4:
            if args.impl == "reference":
                ref = os.path.join(ROOT, "baseline", "_ref")
                if not os.path.isdir(os.path.join(ref, "thundersync")):
                    raise RuntimeError("reference not installed under baseline/_ref")
                sys.path.insert(0, ref)
                model, trainer = build_reference_opd(args, device, world)
            else:
                model, trainer = build_ours_opd(args, device, world)
        elif args.impl == "ours":
            model, trainer = build_ours(args, device)
        else:
            model, trainer = build_reference(args, device)
    except Exception as exc:  # reference unavailable -> one JSON line and exit 0
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": f"{type(exc).__name__}: {exc}"[:300]}))
            return
        raise

    if args.config == 4:
        trainer.open_budget = args.opd_open_trajectories or opd_open_budget(args, device)
        cfg_block["delivery"] = (
            "each action reaches the trainer at its teacher-score arrival time on a clock advanced by the "
            f"trainer's host time per call; the ready actions of distinct trajectories go in one joint "
            f"scored-turn pack (at most {trainer.pack_limit} actions, {trainer.pack_tokens} tokens); same driver for "
            "both arms")
        cfg_block["open_trajectories"] = (
            f"at most {trainer.open_budget} trajectories stream at once per rank (each keeps its K/V and fp32 "
            f"turn-boundary adjoint ledgers on the device until it closes); later trajectories' actions wait in "
            f"arrival order; same budget for both arms")
    extra = (1 if args.profile_out else 0) + (1 if args.cprofile_out else 0)
    mk = make_step_opd if args.config == 4 else make_step
    works = [mk(rank, s, args) for s in range(args.warmup + args.steps + extra)]
    from thundersync_b200.ops import _ext

    for s in range(args.warmup):
        run_step(trainer, works[s], None)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    if args.clocks_file is None:
        args.clocks_file = os.path.join(tempfile.gettempdir(), f"bench_clocks_{os.getpid()}.csv")
    sampler = ClockSampler(args.clocks_file) if rank == 0 else None
    if sampler:
        os.makedirs(os.path.dirname(os.path.abspath(args.clocks_file)), exist_ok=True)
        sampler.start()
    _ext.reset_launch_counts()
    tails = []
    scored_local = 0
    h2d_local = 0
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    wall0 = time.perf_counter()
    start.record()
    issue_s = 0.0
    for s in range(args.warmup, args.warmup + args.steps):
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        h0 = time.perf_counter()
        st = run_step(trainer, works[s], t0)
        issue_s += time.perf_counter() - h0  # host time to issue the step (before its result is read)
        t1.record()
        tails.append((t0, t1))
        scored_local += works[s]["scored"]
        h2d_local += works[s]["tokens"] * 8
        _ = st["global_grad_norm"]  # host read of the step result
    end.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - wall0
    if world > 1:
        dist.barrier()
    clocks = sampler.stop(list(range(world))) if sampler else None
    launches = _ext.launch_counts()["kernels"] if args.impl == "ours" else 0
    dev_ms = start.elapsed_time(end)
    tail_ms = sum(a.elapsed_time(b) for a, b in tails) / len(tails)
    vec = torch.tensor([dev_ms, tail_ms, wall * 1e3, float(scored_local), float(h2d_local)], device=device,
                       dtype=torch.float64)
    if world > 1:
        mx = vec.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = vec.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    else:
        mx, sm = vec, vec
    dev_ms_max, tail_ms_max, wall_ms_max = float(mx[0]), float(mx[1]), float(mx[2])
    scored_total = float(sm[3])
    h2d_total = float(sm[4])
    if rank == 0:
        value = scored_total / (dev_ms_max / 1e3)
        e2e = scored_total / (wall_ms_max / 1e3)
        out = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "scored tokens/s (whole job)",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_ms_max / args.steps, 2),
            "tail_ms": round(tail_ms_max, 2),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None if BASELINE_VALUE is None else round(value / BASELINE_VALUE, 4),
            "dtype": "bf16",
            "data": "synthetic token ids, random-init weights",
            "config": cfg_block,
            "clocks": clocks,
            "e2e": {
                "value": round(e2e, 1),
                "unit": "scored tokens/s (wall clock through the public API)",
                "h2d_bytes_per_step": int(h2d_total / args.steps),
                "d2h_bytes_per_step": 4 * world,
            },
            "gpu_launches": launches,
            "host_issue_ms_per_step": round(issue_s * 1e3 / args.steps, 2),
        }
        if args.impl == "reference":
            out["impl"] = "reference"
            out["gpu_launches"] = 0
            if args.config == 4:
                out["config"]["reference_build"] = {
                    "builder": "thundersync.engine.streaming.StreamingRun(stream_turns=True, turn_boundary_rebuild="
                               "True) + thundersync.opd.objectives.OPDTurnStream, torch AdamW",
                    **reference_diagnostics(),
                }
            else:
                out["config"]["reference_build"] = {
                "builder": "thundersync.grpo.runtime.load_trainer(GrpoTrainerConfig.from_namespace(...))",
                "source_attention_backend": args.ref_attention,
                "compile_pointwise_modules": bool(args.ref_compile),
                "deterministic_algorithms": bool(args.ref_deterministic),
                "optimizer_state_sharding": world > 1,
                "checkpoint": True,
                "statistics": "device_resident sources, statistic_device auto",
                **reference_diagnostics(),
                }
        elif args.config == 4:
            out["config"]["build"] = {"objective": "OPDTurnStream into an fp32 flat gradient",
                                      "optimizer": "fused flat AdamW", "turn_replay": "deferred at close"}
        else:
            out["config"]["build"] = {
                "checkpoint": False,
                "statistics": "device-resident fp32 group statistics",
                "optimizer": "fused flat AdamW" + (" (ZeRO-1 sharded)" if getattr(trainer, "_sharded_flat", False)
                                                   else ""),
            }
        print(json.dumps(out))
    if args.profile_out:
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize()
        with profile(activities=[ProfilerActivity.CPU, ProfilerActivity.CUDA], with_stack=False) as prof:
            run_step(trainer, works[-1], None)
            torch.cuda.synchronize()
        if rank == 0:
            with open(args.profile_out, "w") as fh:
                fh.write(prof.key_averages().table(sort_by="cuda_time_total", row_limit=45,
                                                   max_name_column_width=100))
    if args.cprofile_out:
        import cProfile
        import io
        import pstats

        torch.cuda.synchronize()
        pr = cProfile.Profile()
        t0 = time.perf_counter()
        pr.enable()
        run_step(trainer, works[-1], None)
        pr.disable()
        host_s = time.perf_counter() - t0
        torch.cuda.synchronize()
        total_s = time.perf_counter() - t0
        if rank == 0:
            buf = io.StringIO()
            st = pstats.Stats(pr, stream=buf)
            buf.write(f"host (profiled) {host_s:.3f} s, to device idle {total_s:.3f} s\n")
            st.sort_stats("tottime").print_stats(60)
            st.sort_stats("cumulative").print_stats(60)
            with open(args.cprofile_out, "w") as fh:
                fh.write(buf.getvalue())
    if hasattr(trainer, "shutdown"):
        trainer.shutdown()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
