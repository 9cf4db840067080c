"""Expert-parallel dispatch + combine microbenchmark (forward + backward), one rank per GPU.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        --master-port 29600 bench_ep.py --impl native

Per rank: 8192 tokens, hidden 2048, router logits ~ N(0, 1) over 128 experts, top-8 with
softmax renormalisation, SwiGLU experts (intermediate 768, weights ~ N(0, 0.02)), bf16, seeded.

Two timings per implementation, each the device time (CUDA events on the launching stream,
barrier + synchronize around the timed loop, an L2-flushing 256 MB write between iterations
outside the events) of forward + backward, max over ranks:

* ``dispatch_combine_us``: dispatch -> combine with identity experts (the exchange alone);
* ``moe_layer_us``: dispatch -> grouped SwiGLU experts -> combine.

``nvlink_gbps`` = bytes this rank sends to other GPUs per dispatch+combine forward+backward
(counted from the routing: the native path sends one row per (token, destination rank), the
all-to-all paths one row per (token, expert) pair) / ``dispatch_combine_us``.

``--impl``: ``native`` (this repository's NVLink peer-memory kernels), ``nccl`` (this
repository's all-to-all baseline dispatcher), ``reference`` (the reference package's stock
dispatcher and expert module, installed under baseline/_ref).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--impl", choices=("native", "nccl", "reference"), default="native")
    p.add_argument("--tokens", type=int, default=8192)
    p.add_argument("--hidden", type=int, default=2048)
    p.add_argument("--experts", type=int, default=128)
    p.add_argument("--topk", type=int, default=8)
    p.add_argument("--intermediate", type=int, default=768)
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--reference-experts", choices=("dsv4", "qwen"), default="dsv4",
                   help="reference expert arm: the DeepSeek-V4 RoutedExperts (torch._grouped_mm, fused SwiGLU "
                        "kernel, its own dispatcher) or the Qwen per-expert loop")
    p.add_argument("--kernel-breakdown", default=None, metavar="PREFIX",
                   help="write per-kernel device time of one extra untimed iteration of each arm to "
                        "PREFIX.{exchange,layer}.rankR.json (torch profiler)")
    return p.parse_args(argv)


def _inputs(args, rank, world, dev):
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    x = torch.randn(args.tokens, args.hidden, device=dev, generator=gen, dtype=torch.bfloat16)
    logits = torch.randn(args.tokens, args.experts, device=dev, generator=gen)
    weights, ids = torch.softmax(logits, -1).topk(args.topk, -1)
    weights = weights / weights.sum(-1, keepdim=True)
    dout = torch.randn(args.tokens, args.hidden, device=dev, generator=gen, dtype=torch.bfloat16)
    e_local = args.experts // world
    gen.manual_seed(7 + rank)
    w1 = (torch.randn(e_local, 2 * args.intermediate, args.hidden, device=dev, generator=gen) * 0.02).bfloat16()
    w2 = (torch.randn(e_local, args.hidden, args.intermediate, device=dev, generator=gen) * 0.02).bfloat16()
    return x, weights, ids.to(torch.int32), dout, w1, w2


def _sent_bytes(ids, e_local, rank, world, hidden, dedupe):
    owners = (ids.long() // e_local)
    if dedupe:
        dest = torch.zeros(ids.shape[0], world, dtype=torch.bool, device=ids.device)
        dest.scatter_(1, owners, True)
        remote = int(dest.sum()) - int(dest[:, rank].sum())
    else:
        remote = int((owners != rank).sum())
    return 4 * remote * hidden * 2  # dispatch + combine, forward + backward


def _native_step(args, mesh, tensors, experts):
    from tiny_dsv41_b200.ops import gemm as G
    from tiny_dsv41_b200.ops import moe as M
    from tiny_dsv41_b200.parallel.dispatch import AllToAllTokenDispatcher
    from tiny_dsv41_b200.parallel.nvlink_ep import NVLinkTokenDispatcher

    cls = NVLinkTokenDispatcher if args.impl == "native" else AllToAllTokenDispatcher
    disp = cls(mesh, max_tokens=args.tokens) if cls is NVLinkTokenDispatcher else cls(mesh)
    disp.expert_range(args.experts)
    x, weights, ids, dout, w1, w2 = tensors

    def step():
        xa = x.detach().requires_grad_()
        wa = weights.detach().requires_grad_()
        batch = disp.dispatch(xa, ids, wa)
        if experts:
            gu = G.grouped_linear(batch.rows, w1, batch.offsets, batch.sizes)
            act = M.swiglu(gu, total=batch.total)
            y = G.grouped_linear(act, w2, batch.offsets, batch.sizes)
        else:
            y = batch.rows
        out = disp.combine(y, batch, weighted=True)
        out.backward(dout)

    return step


def _reference_dsv4_experts(args, mesh, w1, w2, device):
    """The reference's DeepSeek-V4 routed experts on its own dispatcher: dispatch, grouped GEMMs on
    ``torch._grouped_mm``, its SwiGLU x route-weight kernel, combine. The config object carries only
    the fields the module reads; the SwiGLU clamp is set beyond any activation (the benchmark's
    experts are plain SwiGLU)."""
    from types import SimpleNamespace

    from dsv41_train.models.dsv4.moe.dispatch import AllToAllTokenDispatcher as Dsv4Dispatcher
    from dsv41_train.models.dsv4.moe.module import RoutedExperts

    cfg = SimpleNamespace(n_routed_experts=args.experts, hidden_size=args.hidden,
                          moe_intermediate_size=args.intermediate, swiglu_limit=1.0e30)
    module = RoutedExperts(cfg, Dsv4Dispatcher(mesh)).to(device=device, dtype=torch.bfloat16)
    e = module.num_experts
    with torch.no_grad():  # same expert weights as the other arms: [E, 2I, H] gate rows then up rows
        module.gate_up.copy_(w1.view(e, 2, args.intermediate, args.hidden).transpose(1, 2))
        module.down.copy_(w2)
    return module


def _reference_step(args, mesh, tensors, experts):
    sys.path.append(os.path.join(ROOT, "baseline", "_ref"))
    from dsv41_train.dispatch import AllToAllTokenDispatcher
    from dsv41_train.models.qwen.config import Qwen3MoeConfig
    from dsv41_train.models.qwen.model import Qwen3MoeExperts

    disp = AllToAllTokenDispatcher(mesh)
    x, weights, ids, dout, w1, w2 = tensors
    module = None
    if experts and getattr(args, "reference_experts", "dsv4") == "dsv4":
        module = _reference_dsv4_experts(args, mesh, w1, w2, x.device)
    elif experts:
        cfg = Qwen3MoeConfig(hidden_size=args.hidden, moe_intermediate_size=args.intermediate,
                             num_experts=args.experts, num_experts_per_tok=args.topk)
        module = Qwen3MoeExperts(cfg, disp).to(x.device)
        with torch.no_grad():
            module.gate_up_proj.data = w1.clone()
            module.down_proj.data = w2.clone()
    else:
        disp.expert_range(args.experts)
    ids_long = ids.long()

    def step():
        xa = x.detach().requires_grad_()
        wa = weights.detach().requires_grad_()
        if module is not None:
            out = module(xa, ids_long, wa)
        else:
            hidden, _, routed_w, meta = disp.dispatch(xa, ids_long, wa)
            out = disp.combine(hidden * routed_w[:, None].to(hidden.dtype), meta)
        out.backward(dout)

    return step


def _time(step, args, dev, census_path=None):
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    for _ in range(args.warmup):
        step()
    if census_path:  # one extra untimed iteration under the profiler, before the timed loop
        from tiny_dsv41_b200.utils.kernel_census import kernel_census, write_census

        dist.barrier()
        write_census(kernel_census(step), census_path, rank=dist.get_rank(), world=dist.get_world_size())
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.iters)]
    dist.barrier()
    torch.cuda.synchronize()
    for start, end in events:
        flush.zero_()
        start.record()
        step()
        end.record()
    dist.barrier()
    torch.cuda.synchronize()
    total_ms = sum(s.elapsed_time(e) for s, e in events)
    t = torch.tensor([total_ms / args.iters * 1000.0], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def main(argv=None) -> None:
    args = parse_args(argv)
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    from torch.distributed.device_mesh import init_device_mesh

    mesh = init_device_mesh("cuda", (world,), mesh_dim_names=("ep",))
    tensors = _inputs(args, rank, world, dev)
    make = _reference_step if args.impl == "reference" else _native_step
    try:
        kb = args.kernel_breakdown
        comm_us = _time(make(args, mesh, tensors, False), args, dev, kb and f"{kb}.exchange.rank{rank}.json")
        layer_us = _time(make(args, mesh, tensors, True), args, dev, kb and f"{kb}.layer.rank{rank}.json")
        sent = _sent_bytes(tensors[2], args.experts // world, rank, world, args.hidden, args.impl == "native")
        b = torch.tensor([float(sent)], device=dev)
        dist.all_reduce(b, op=dist.ReduceOp.MAX)
        result = {"metric": "EP dispatch+combine fwd+bwd (max over ranks)", "impl": args.impl, "ep": world,
                  "tokens_per_rank": args.tokens, "hidden": args.hidden, "experts": args.experts, "topk": args.topk,
                  "dispatch_combine_us": round(comm_us, 1), "moe_layer_us": round(layer_us, 1),
                  "bytes_sent_per_rank": int(b.item()), "nvlink_gbps": round(b.item() / (comm_us * 1e-6) / 1e9, 1),
                  "dtype": "bf16", "data": "seeded synthetic", "timing": "CUDA events, L2 flushed between iterations"}
    except Exception as error:  # pragma: no cover - the reference arm may not run here
        if args.impl != "reference":
            raise
        result = {"impl": "reference", "unavailable": f"{type(error).__name__}: {error}"[:300]}
    if rank == 0:
        print(json.dumps(result), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
