"""Qwen3-MoE full-parameter trainer (the public training API) and its benchmark harness.

:class:`QwenTrainer` builds the model directly on the GPU (meta-device construction, then
random init on the device), places experts with EP, keeps dense weights as bf16 replicas whose
fp32 master and AdamW moments are sharded over the world (``parallel/peer_fsdp.py``: one NVLink
kernel per layer reduces the gradient, updates the shard and writes the new weights to every
rank; ``dense_sync="fsdp"`` selects FSDP2 over NCCL instead), and applies AdamW with fp32 master
weights inside the backward pass.
``train_step(input_ids, labels)`` is one optimizer step; inputs may live on the host (pinned) or
the device.

:class:`QwenSFTBench` times it the way ``bench.py`` reports: device time of exactly K steps
(CUDA events, barrier + synchronize on both sides, max over ranks) and an end-to-end wall time
through ``train_step`` including the per-step host-to-device input copy and loss read-back.
"""

from __future__ import annotations

import os
import time
import zlib

import torch
import torch.distributed as dist

from ..ops import StatusMonitor

from ..models.qwen import Qwen3MoeConfig, Qwen3MoeForCausalLM
from ..models.qwen.model import Qwen3MoeExperts
from ..optim import FusedAdamW
from ..parallel.cp import ContextParallel
from ..parallel.dispatch import AllToAllTokenDispatcher, TokenDispatcher
from ..runtime import initialize_runtime


def _init_on_device(model: Qwen3MoeForCausalLM, seed: int, rank: int) -> None:
    gen = torch.Generator(device="cuda")
    std = model.config.initializer_range
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm.weight") or "layernorm" in name:
                p.fill_(1.0)
            elif name.endswith("bias"):
                p.zero_()
            else:
                is_expert = ".experts." in name
                gen.manual_seed(seed + (1000003 * (rank + 1) if is_expert else 0) + zlib.crc32(name.encode()) % 100003)
                p.normal_(0.0, std, generator=gen)


class QwenTrainer:
    def __init__(self, config: Qwen3MoeConfig, *, lr: float = 1e-5, moment_dtype=torch.float32,
                 dispatcher: str = "auto", gradient_checkpointing: bool = True, seed: int = 0,
                 tokens_per_rank: int = 4096, cp_size: int = 1, dense_sync: str = "auto",
                 cuda_graph: bool = False, graph_warmup: int = 2) -> None:
        self.runtime = initialize_runtime(require_distributed=int(os.environ.get("WORLD_SIZE", "1")) > 1,
                                          timeout_seconds=900)
        rt = self.runtime
        torch.manual_seed(seed)
        self.world = rt.world_size
        self.tokens_per_rank = tokens_per_rank  # sizes the NVLink receive slabs
        self.cp_size = cp_size
        self.meshes = None
        cp = ContextParallel()
        if self.world > 1:
            from ..parallel.meshes import ParallelMeshes

            self.meshes = ParallelMeshes.build(cp=cp_size, ep=self.world)
            if cp_size > 1:  # each sequence split in cp contiguous chunks; K/V exchanged inside attention
                cp = ContextParallel(self.meshes.cp)
            token_dispatcher = self._make_dispatcher(dispatcher)
        else:
            token_dispatcher = TokenDispatcher()
        self.dispatcher = token_dispatcher
        with torch.device("meta"):
            model = Qwen3MoeForCausalLM(config, cp, token_dispatcher)
        model = model.to_empty(device=rt.device).to(torch.bfloat16)
        _init_on_device(model, seed, rt.rank)
        if gradient_checkpointing:
            model.gradient_checkpointing_enable()
        model.train()
        self.expert_params = [p for m in model.modules() if isinstance(m, Qwen3MoeExperts) for p in m.parameters()]
        expert_ids = {id(p) for p in self.expert_params}
        # dense weights: "peer" = bf16 replicas with a sharded optimizer fused with the gradient
        # reduce-scatter and the parameter all-gather over NVLink (parallel/peer_fsdp.py);
        # "fsdp" = FSDP2 over NCCL (the reference's scheme)
        if dense_sync == "auto":
            dense_sync = "peer" if rt.device.type == "cuda" else ("fsdp" if self.world > 1 else "local")
        self.dense_sync = dense_sync if self.world > 1 or dense_sync == "peer" else "local"
        if self.world > 1 and self.dense_sync == "fsdp":
            self._apply_fsdp(model)
        self.model = model
        # device status word (bounded peer waits, bounds checks) read once per step by the loops
        self.monitor = StatusMonitor(rt.device)
        hyper = dict(lr=lr, betas=(0.9, 0.95), weight_decay=0.1, moment_dtype=moment_dtype)
        # in-backward updates on side streams (TDSV_SIDE_STREAM=0 keeps them on the compute stream;
        # TDSV_SIDE_BLOCKS caps the CTAs of the expert update running beside the backward GEMMs)
        side = rt.device.type == "cuda" and os.environ.get("TDSV_SIDE_STREAM", "1") != "0"
        side_blocks = int(os.environ.get("TDSV_SIDE_BLOCKS", "0"))
        if self.dense_sync == "peer":
            from ..parallel.peer_fsdp import PeerShardedOptimizer, decoder_units

            dense_opt = PeerShardedOptimizer(decoder_units(model, expert_ids), algo="adamw", **hyper)
        else:
            dense = [p for p in model.parameters() if id(p) not in expert_ids]
            # under FSDP the update follows FSDP's own reduce-scatter stream; it stays on the default stream
            dense_opt = FusedAdamW(dense, in_backward=True, side_stream=side and self.dense_sync != "fsdp", **hyper)
        self.optimizers = [
            dense_opt,
            FusedAdamW(self.expert_params, in_backward=True, grad_scale=1.0 / self.world, side_stream=side,
                       side_blocks=side_blocks, **hyper),
        ]
        # CUDA graph of a whole training step (forward, backward, in-backward optimizer, NVLink
        # exchanges): captured after `graph_warmup` eager steps, then replayed. Every per-step value a
        # kernel needs (exchange epochs, step counts) lives in device memory and advances inside the
        # graph, so a replay is one launch from the host instead of several thousand.
        self.cuda_graph = bool(cuda_graph) and rt.device.type == "cuda"
        if self.cuda_graph and (cp_size > 1 or self.dense_sync == "fsdp"):
            raise ValueError("CUDA-graph steps need cp_size 1 and dense_sync 'peer' (no NCCL inside the step)")
        self.graph_warmup = graph_warmup
        self._eager_steps = 0
        self._graph = None

    def _make_dispatcher(self, kind: str):
        if kind in ("auto", "nvlink"):
            try:
                from ..parallel.nvlink_ep import NVLinkTokenDispatcher

                return NVLinkTokenDispatcher(self.meshes.ep, max_tokens=self.tokens_per_rank)
            except ImportError:
                if kind == "nvlink":
                    raise
        return AllToAllTokenDispatcher(self.meshes.ep)

    def _apply_fsdp(self, model) -> None:
        from torch.distributed.fsdp import MixedPrecisionPolicy, fully_shard

        policy = MixedPrecisionPolicy(param_dtype=torch.bfloat16, reduce_dtype=torch.float32)
        # dense weights are sharded over every rank: under context parallelism the ranks of a CP
        # group hold different tokens of one sequence, so their gradients are reduced together
        # (the CP mean loss scales its backward by cp, which makes the world average exact)
        mesh = self.meshes.world
        ignored = set(self.expert_params)
        # Decoder layers stay gathered from their forward to their backward: 48 layers of bf16 attention
        # and router weights are ~1.8 GB, and this saves the second all-gather per layer (the
        # recompute and the backward reuse the forward's copy).
        opts = {"mesh": mesh, "mp_policy": policy, "reshard_after_forward": True}
        fully_shard(model.model.embed_tokens, **opts)
        for layer in model.model.layers:
            fully_shard(layer, ignored_params=ignored, **{**opts, "reshard_after_forward": False})
        fully_shard(model.lm_head, **opts)
        # the root keeps its parameters gathered between forward and backward (FSDP2's default
        # for a root): its output is a dataclass, so no pre-backward hook could re-gather them
        fully_shard(model, mesh=mesh, mp_policy=policy, ignored_params=ignored)
        # MoE layers issue EP exchanges on their own group in backward; an implicit cross-layer
        # all-gather prefetch could interleave the two groups' collectives differently on
        # different ranks, so each FSDP module prefetches nothing but itself.
        from torch.distributed.fsdp import FSDPModule

        for module in model.modules():
            if isinstance(module, FSDPModule):
                module.set_modules_to_backward_prefetch([module])

    def train_step(self, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """One optimizer step; returns the loss as a device scalar (inputs on the host or device)."""
        if self._graph is not None:
            self._static_ids.copy_(input_ids, non_blocking=True)
            self._static_labels.copy_(labels, non_blocking=True)
            self._graph.replay()
            return self._static_loss
        if self.cuda_graph and self._eager_steps >= self.graph_warmup:
            return self._capture(input_ids, labels)
        device = self.runtime.device
        loss = self._step(input_ids.to(device, non_blocking=True), labels.to(device, non_blocking=True))
        self._eager_steps += 1
        return loss

    def _step(self, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        for opt in self.optimizers:
            opt.begin_step()
        out = self.model(input_ids, labels=labels, output_router_logits=True)
        out.loss.backward()
        for opt in self.optimizers:
            opt.finish_step()
        self.dispatcher.end_step()
        return out.loss.detach()

    def _capture(self, input_ids: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """Capture one step into a CUDA graph (nothing runs during capture), then run it once."""
        import gc

        device = self.runtime.device
        self._static_ids = torch.empty(input_ids.shape, dtype=input_ids.dtype, device=device)
        self._static_labels = torch.empty(labels.shape, dtype=labels.dtype, device=device)
        self._static_ids.copy_(input_ids, non_blocking=True)
        self._static_labels.copy_(labels, non_blocking=True)
        torch.cuda.synchronize(device)
        gc.collect()
        torch.cuda.empty_cache()  # eager-step blocks go back, the graph's private pool takes their place
        graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(graph):
                loss = self._step(self._static_ids, self._static_labels)
        except RuntimeError as error:
            # Nothing ran during the failed capture, and an eager step issues the same kernels in the
            # same order with the same device-side epochs, so this rank can carry on eagerly even if
            # its peers replay graphs.
            import warnings

            warnings.warn(f"CUDA-graph capture failed, continuing with eager steps: {error}")
            del graph
            self.cuda_graph = False
            torch.cuda.synchronize(device)
            for opt in self.optimizers:  # the capture's Python-side bookkeeping is rolled back
                if hasattr(opt, "_inflight"):
                    opt._inflight.clear()
            self.dispatcher.abort_step()
            loss = self._step(self._static_ids, self._static_labels)
            self._eager_steps += 1
            return loss
        self._graph, self._static_loss = graph, loss
        graph.replay()
        return loss

    def close(self) -> None:
        self._graph = None
        for opt in self.optimizers:
            opt.remove_hooks()
        if dist.is_initialized():
            dist.barrier()
            dist.destroy_process_group()


class QwenSFTBench:
    def __init__(self, args) -> None:
        self.args = args
        config = Qwen3MoeConfig(num_hidden_layers=args.layers, max_window_layers=args.layers)
        moment = torch.float32 if args.moment_dtype == "fp32" else torch.bfloat16
        self.cp = getattr(args, "cp", 1)
        self.trainer = QwenTrainer(config, lr=args.lr, moment_dtype=moment, dispatcher=args.dispatcher,
                                   tokens_per_rank=args.batch_size * args.seq_len // self.cp, cp_size=self.cp,
                                   dense_sync=getattr(args, "dense_sync", "auto"),
                                   cuda_graph=getattr(args, "cuda_graph", False))
        self.config = config

    def _batch(self, gen: torch.Generator):
        a = self.args
        ids = torch.randint(0, self.config.vocab_size, (a.batch_size, a.seq_len), generator=gen)
        ids[:, 0] = self.config.bos_token_id
        labels = ids.clone()
        labels[:, : a.seq_len // 2] = -100  # loss on the last 50% of tokens
        return ids.pin_memory(), labels.pin_memory()

    def _count_launches(self, batches) -> dict:
        """Kernels launched in one (extra, untimed) step, split into this repo's and others."""
        from ..utils.kernel_census import kernel_census, write_census

        ids, labels = batches[0]
        census = kernel_census(lambda: self.trainer.train_step(ids, labels))
        path = getattr(self.args, "kernel_breakdown", None)
        if path and self.trainer.runtime.rank == 0:
            write_census(census, path, rank=0, world=self.trainer.world)
        return {"own": census["own"], "other": census["other"]}

    def run(self) -> dict:
        import sys

        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
        from bench import ClockSampler

        a = self.args
        t = self.trainer
        rt = t.runtime
        # the ranks of one CP group train on the same sequences (each keeps its own chunk)
        gen = torch.Generator().manual_seed(1234 + rt.rank // self.cp)
        batches = [self._batch(gen) for _ in range(4)]
        # L2 flush buffer (larger than the 126 MB L2) written between timed steps
        flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=rt.device)
        for i in range(a.warmup):
            t.train_step(*batches[i % len(batches)])
        torch.cuda.synchronize()

        def barrier():
            if dist.is_initialized():
                dist.barrier()
            torch.cuda.synchronize()

        # device-timed region: exactly K steps
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        losses = []
        with ClockSampler(rt.local_rank) as clocks:
            barrier()
            start.record()
            host0 = time.perf_counter()
            for i in range(a.steps):
                flush.zero_()
                losses.append(t.train_step(*batches[i % len(batches)]))
            end.record()
            host_ms = (time.perf_counter() - host0) * 1000.0  # time to enqueue the K steps (no sync inside)
            barrier()
        device_ms = start.elapsed_time(end)
        t.monitor.step_end("timed steps")
        # end-to-end through the public API: H2D of inputs, D2H of the loss every step
        barrier()
        wall0 = time.perf_counter()
        e2e_losses = []
        for i in range(a.steps):
            loss = t.train_step(*batches[i % len(batches)])
            e2e_losses.append(loss.item())
            t.monitor.step_end("train_step")
        torch.cuda.synchronize()
        wall_s = time.perf_counter() - wall0
        peak_gib = torch.cuda.max_memory_allocated(rt.device) / 2 ** 30
        # kernel census of one more (untimed) step of the same shape; after the timed loops, so the
        # profiler's instrumentation cannot touch them
        launches = self._count_launches(batches)
        times = torch.tensor([device_ms, wall_s * 1000.0, peak_gib, host_ms], device=rt.device)
        if dist.is_initialized():
            dist.all_reduce(times, op=dist.ReduceOp.MAX)
        device_ms, wall_ms, peak_gib, host_ms = times.tolist()
        tokens = a.batch_size * a.seq_len * (rt.world_size // self.cp) * a.steps
        value = tokens / (device_ms / 1000.0)
        e2e = tokens / (wall_ms / 1000.0)
        final_loss = float(losses[-1].item())
        return {
            "value": value,
            "ms_per_step": device_ms / a.steps,
            "e2e": {"value": e2e, "unit": "tokens/s", "ms_per_step": wall_ms / a.steps,
                    "h2d_bytes_per_step": 2 * a.batch_size * a.seq_len * 8, "d2h_bytes_per_step": 4},
            "gpu_launches": launches["own"] * a.steps,
            "other_launches_per_step": launches["other"],
            "loss": final_loss,
            "e2e_last_loss": e2e_losses[-1],
            "peak_memory_gib": round(peak_gib, 2),
            "host_enqueue_ms_per_step": round(host_ms / a.steps, 1),
            "clocks": clocks.summary(),
            "config": {
                "model": MODEL_NAME if self.config.num_hidden_layers == 48 else f"REDUCED {self.config.num_hidden_layers}L (not the benchmark)",
                "global_batch": a.batch_size * rt.world_size // self.cp, "seq_len": a.seq_len,
                "parallelism": ((f"cp{self.cp}+" if self.cp > 1 else "") + f"ep{rt.world_size}+"
                                + ("dp" if t.dense_sync == "peer" else "fsdp") + f"{rt.world_size}"
                                if rt.world_size > 1 else "single-gpu"),
                "optimizer": f"AdamW in-backward, fp32 master, {a.moment_dtype} moments",
                "dense_sync": t.dense_sync,
                "cuda_graph": t._graph is not None,
                "grad_ckpt": True, "l2": "256 MB buffer written between timed steps",
                "loss_tokens": "last 50%",
            },
        }

    def close(self) -> None:
        self.trainer.close()


MODEL_NAME = "Qwen3-30B-A3B-shaped (48L, H2048, 32q/4kv x128, 128 experts top-8, I768, V151936)"
