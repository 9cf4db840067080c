"""Headline benchmark: Qwen3-30B-A3B-shaped full SFT step, tokens/s for the whole job.

Config: 48 layers, hidden 2048, 32 q / 4 kv heads, head_dim 128, RoPE theta
1e6, 128 experts top-8 with intermediate 768, vocab 151936; seq 4096, batch 1 per rank,
uniform-random token ids (synthetic), loss on the last 50% of tokens, random-init (std 0.02),
AdamW with fp32 master weights, gradient checkpointing, EP = N (+ FSDP = N for dense weights).

    python bench.py --gpus N --steps K --warmup W                 # native arm
    python bench.py --impl reference --gpus N --steps K --warmup W  # unmodified reference arm

For N > 1 launch with ``python -m torch.distributed.run --nproc-per-node N ... bench.py``.
Rank 0 prints one JSON line. The device-timed ``value`` brackets exactly K steps with a barrier
and ``torch.cuda.synchronize()`` on both sides and takes the max over ranks; the ``e2e`` value
times the same steps through the public training API including the pinned host-to-device copy of
each step's tokens and the device-to-host read of its loss.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "SFT tokens/sec/box (max over ranks)"
MODEL = "Qwen3-30B-A3B-shaped (48L, H2048, 32q/4kv x128, 128 experts top-8, I768, V151936)"
# The reference publishes no B200 or Qwen number; its only published SFT throughput is for
# DeepSeek-V4.1-Flash on 8x B300 (docs/testing.md there), a different model, so vs_baseline stays null.
BASELINE_VALUE = None


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=("native", "reference"), default="native")
    p.add_argument("--seq-len", type=int, default=4096)
    p.add_argument("--batch-size", type=int, default=1)
    p.add_argument("--cp", type=int, default=1,
                   help="context-parallel degree (BASELINE config 4: --cp 2 --seq-len 32768 on 4 GPUs, EP = N)")
    p.add_argument("--layers", type=int, default=48, help="development only: fewer layers is not the benchmark")
    p.add_argument("--dispatcher", choices=("auto", "nccl", "nvlink"), default="auto")
    p.add_argument("--moment-dtype", choices=("auto", "fp32", "bf16"), default="auto",
                   help="auto: fp32 AdamW moments when they fit in HBM at this N, else bf16")
    p.add_argument("--lr", type=float, default=1e-5)
    p.add_argument("--dense-sync", choices=("auto", "peer", "fsdp"), default="auto",
                   help="dense weights: peer = bf16 replicas + sharded AdamW fused with the NVLink gradient "
                        "reduce-scatter and parameter gather (default on GPUs); fsdp = FSDP2 over NCCL")
    p.add_argument("--cuda-graph", action=argparse.BooleanOptionalAction, default=None,
                   help="replay each training step as one captured CUDA graph (default: on when the step "
                        "has no NCCL call, i.e. --cp 1 and peer dense sync)")
    p.add_argument("--kernel-breakdown", default=None, metavar="FILE",
                   help="write per-kernel device time of one extra untimed step (torch profiler) as JSON")
    args = p.parse_args(argv)
    if args.cuda_graph is None:
        args.cuda_graph = args.cp == 1 and args.dense_sync != "fsdp"
    return args


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons while the timed region runs.

    One long-lived ``nvidia-smi -lms 200`` child started on entry and stopped on exit: sampling
    from a thread with one ``subprocess.run`` per sample would fork this (large) process every
    200 ms and take the interpreter lock from the thread that launches the kernels."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int) -> None:
        self.index = index
        self.samples: list[list[str]] = []
        self._proc = None

    def __enter__(self):
        import tempfile

        self._log = tempfile.NamedTemporaryFile(prefix="clocks-", suffix=".csv", delete=False)
        self._log.close()
        try:
            self._proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                           "--format=csv,noheader,nounits", "-lms", "200", "-f", self._log.name],
                                          stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except OSError:
            self._proc = None
        return self

    def __exit__(self, *exc):
        import signal

        if self._proc is None:
            return
        self._proc.send_signal(signal.SIGINT)  # the loop mode's own stop request: flushes the log
        try:
            self._proc.wait(timeout=10)
        except subprocess.TimeoutExpired:
            self._proc.kill()
            self._proc.wait()
        try:
            with open(self._log.name) as f:
                out = f.read()
        finally:
            os.unlink(self._log.name)
        for line in out.strip().splitlines():
            fields = [x.strip() for x in line.split(",")]
            if len(fields) >= 9:
                self.samples.append(fields)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = sorted(float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit())
        mx = max((float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()), default=None)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if len(s) > 5 + i and s[5 + i] == "Active"})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": reasons,
                "samples": len(self.samples)}


def emit(record: dict) -> None:
    print(json.dumps(record), flush=True)


HBM_BYTES = 178 * 2 ** 30       # usable B200 capacity reported by torch
ACTIVATION_RESERVE = 24 * 2 ** 30  # recompute transients, logits, NVLink slabs, replay records, allocator slack


def memory_plan(args, world: int) -> tuple[bool, str]:
    """Whether the persistent training state fits in HBM at this N, choosing the moment dtype when
    ``--moment-dtype auto``: bf16 params + fp32 master + fp32 (or bf16) AdamW moments per parameter.
    Gradients are transient (the optimizer runs inside the backward pass)."""
    from tiny_dsv41_b200.models.qwen import Qwen3MoeConfig

    cfg = Qwen3MoeConfig(num_hidden_layers=args.layers, max_window_layers=args.layers)
    experts = cfg.num_hidden_layers * cfg.num_experts * 3 * cfg.hidden_size * cfg.moe_intermediate_size
    dense = (cfg.num_hidden_layers * (cfg.hidden_size * (cfg.num_attention_heads + 2 * cfg.num_key_value_heads)
                                      * cfg.head_dim * 2 + cfg.hidden_size * cfg.num_experts)
             + 2 * cfg.vocab_size * cfg.hidden_size)
    per_rank = experts / world + dense / world
    budget = HBM_BYTES - ACTIVATION_RESERVE
    choices = ("fp32", "bf16") if args.moment_dtype == "auto" else (args.moment_dtype,)
    # dense weights kept as bf16 replicas with a staged gradient copy (peer-memory sync) instead of shards
    replicas = dense * 4 - dense / world * 2 if getattr(args, "dense_sync", "auto") != "fsdp" else 0.0
    for moments in choices:
        need = per_rank * (2 + 4 + (8 if moments == "fp32" else 4)) + replicas
        if need <= budget:
            args.moment_dtype = moments
            return True, f"{need / 2 ** 30:.0f} GiB of persistent state per rank ({moments} moments)"
    return False, (f"{(experts + dense) / 1e9:.1f}B params; {per_rank / 1e9:.2f}B per rank x "
                   f"{2 + 4 + (8 if choices[-1] == 'fp32' else 4)} B (bf16 param, fp32 master, {choices[-1]} moments) "
                   f"= {need / 2 ** 30:.0f} GiB > {budget / 2 ** 30:.0f} GiB of HBM left after activations per B200")


def run_native(args) -> None:
    # grow allocator segments in place instead of new cudaMalloc calls (which synchronise the device)
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    import torch
    import torch.distributed as dist

    from tiny_dsv41_b200.train.qwen_sft import QwenSFTBench

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    fits, why = memory_plan(args, world)
    base = {"metric": METRIC, "impl": "native", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "dtype": "bf16", "data": "synthetic",
            "unit": "tokens/s"}
    if not fits:
        if rank == 0:
            emit({**base, "value": None, "unavailable": f"full config does not fit: {why}", "vs_baseline": None,
                  "config": {"model": MODEL, "seq_len": args.seq_len, "global_batch": args.batch_size * world}})
        return
    try:
        bench = QwenSFTBench(args)
        result = bench.run()
    except torch.OutOfMemoryError as error:
        # every rank reaches here or fails its next collective within the process-group timeout
        if rank == 0:
            emit({**base, "value": None, "vs_baseline": None,
                  "unavailable": f"out of GPU memory at N={world}: {str(error).splitlines()[0][:200]}",
                  "config": {"model": MODEL, "seq_len": args.seq_len, "cp": args.cp}})
        return
    if rank == 0:
        record = {**base, **result}
        record["vs_baseline"] = (None if BASELINE_VALUE is None or record.get("value") is None
                                 else record["value"] / BASELINE_VALUE)
        emit(record)
    bench.close()


def run_reference(args) -> None:
    sys.path.insert(0, os.path.join(ROOT, "baseline", "_ref"))
    from tiny_dsv41_b200.train.reference_arm import run_reference_arm

    record = run_reference_arm(args, METRIC, MODEL)
    if record is not None and int(os.environ.get("RANK", "0")) == 0:
        emit(record)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_native(args)


if __name__ == "__main__":
    main()
