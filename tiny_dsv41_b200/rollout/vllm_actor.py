"""An owned vLLM engine in a child process: rollouts for Qwen-family policies whose trainable part
is the LM head (the reference's Qwen-head profile, ``rollout_manager/backends/vllm_actor.py``,
``vllm_controller.py``, ``vllm_worker.py``).

* :class:`VLLMActor` (learner side) spawns the child, which builds the engine once and answers
  requests over a pipe: ``generate`` (token-id prompts -> sampled token ids and their log-probs),
  ``update_head`` (new LM-head weights with a version), ``receipt`` and ``close``.
* The child serves one request at a time, so an update always lands between generations (the
  engine is drained); after loading, it reads the weights back from the device and returns their
  SHA-256 with the version, and the learner checks that digest against the one it computed from
  what it sent.
* The engine is created by a factory named ``"module:attribute"`` (imported in the child). The
  default, :class:`VLLMHeadEngine`, drives ``vllm.LLM``: prompts as token ids, one sampling seed
  per request, and head updates through ``LLM.collective_rpc`` on every worker. Tests pass a fake
  factory, so the protocol runs without vLLM or a GPU.
"""

from __future__ import annotations

import hashlib
import importlib
import multiprocessing as mp
import time
import traceback
from dataclasses import dataclass

import torch


def tensor_digest(weight: torch.Tensor) -> str:
    """SHA-256 of a tensor's bytes (bf16 as stored), the identity of a head update."""
    data = weight.detach().to("cpu").contiguous()
    return hashlib.sha256(data.view(torch.uint8).numpy().tobytes()).hexdigest()


@dataclass(frozen=True)
class GenerationRequest:
    prompts: list            # list of token-id lists
    max_tokens: int
    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    seed: int = 0
    stop_token_ids: tuple = ()


def _set_head(worker, weight):  # runs inside each vLLM worker (collective_rpc)
    model = worker.model_runner.model
    head = model.lm_head.weight
    head.data.copy_(weight.to(device=head.device, dtype=head.dtype))
    return tensor_digest(head.data)


class VLLMHeadEngine:
    """``vllm.LLM`` with token-id prompts and LM-head replacement (the default engine)."""

    def __init__(self, settings: dict) -> None:
        from vllm import LLM

        self.llm = LLM(model=settings["model_dir"], dtype="bfloat16", seed=int(settings.get("seed", 0)),
                       gpu_memory_utilization=float(settings.get("gpu_memory_utilization", 0.5)),
                       max_model_len=int(settings.get("max_model_len", 4096)),
                       enforce_eager=bool(settings.get("enforce_eager", False)),
                       tensor_parallel_size=int(settings.get("tensor_parallel_size", 1)))

    def generate(self, request: GenerationRequest) -> list[dict]:
        from vllm import SamplingParams
        from vllm.inputs import TokensPrompt

        outputs = []
        for index, prompt in enumerate(request.prompts):
            params = SamplingParams(temperature=request.temperature, top_p=request.top_p,
                                    top_k=request.top_k if request.top_k > 0 else -1, max_tokens=request.max_tokens,
                                    seed=request.seed + index, logprobs=0,
                                    stop_token_ids=list(request.stop_token_ids))
            done = self.llm.generate([TokensPrompt(prompt_token_ids=list(prompt))], params, use_tqdm=False)[0]
            completion = done.outputs[0]
            logprobs = [float(step[token].logprob) for step, token in zip(completion.logprobs or [],
                                                                           completion.token_ids)]
            outputs.append({"token_ids": list(completion.token_ids), "log_probs": logprobs,
                            "finish_reason": completion.finish_reason})
        return outputs

    def load_head(self, weight: torch.Tensor) -> list[str]:
        return list(self.llm.collective_rpc(_set_head, args=(weight,)))

    def close(self) -> None:
        del self.llm


def _resolve(path: str):
    module, _, attribute = path.partition(":")
    return getattr(importlib.import_module(module), attribute)


def _actor_main(connection, settings: dict) -> None:
    """Child: build the engine, then serve one request at a time until ``close``."""
    try:
        engine = _resolve(settings["engine"])(settings)
        state = {"version": -1, "digest": None}
        connection.send({"id": 0, "value": {"ready": True, **state}})
        while True:
            request = connection.recv()
            command = request["command"]
            if command == "generate":
                value = engine.generate(request["request"])
            elif command == "update_head":
                digests = engine.load_head(request["weight"])
                if len(set(digests)) != 1:
                    raise RuntimeError("workers disagree on the loaded head")
                state = {"version": int(request["version"]), "digest": digests[0]}
                value = dict(state)
            elif command == "receipt":
                value = dict(state)
            elif command == "close":
                engine.close()
                connection.send({"id": request["id"], "value": {"closed": True, **state}})
                return
            else:
                raise ValueError(f"unknown actor command {command!r}")
            connection.send({"id": request["id"], "value": value})
    except BaseException:
        try:
            connection.send({"fatal": traceback.format_exc()})
        except (BrokenPipeError, EOFError, OSError):
            pass
    finally:
        connection.close()


class VLLMActor:
    """Learner-side handle of the owned engine process (see the module docstring)."""

    def __init__(self, model_dir: str, *, engine: str = "tiny_dsv41_b200.rollout.vllm_actor:VLLMHeadEngine",
                 timeout: float = 600.0, **engine_settings) -> None:
        self.settings = {"model_dir": str(model_dir), "engine": engine, **engine_settings}
        self.timeout = timeout
        self.process = None
        self.connection = None
        self.counter = 0
        self.failed = False
        self.head = {"version": -1, "digest": None}

    def _reply(self, request_id: int):
        deadline = time.monotonic() + self.timeout
        while True:
            left = deadline - time.monotonic()
            if left <= 0:
                self.failed = True
                raise TimeoutError("vLLM actor did not answer in time")
            if self.connection.poll(min(left, 0.1)):
                try:
                    message = self.connection.recv()
                except EOFError:
                    self.failed = True
                    raise RuntimeError("vLLM actor closed its channel") from None
                if "fatal" in message:
                    self.failed = True
                    raise RuntimeError("vLLM actor failed:\n" + message["fatal"])
                if message["id"] != request_id:
                    self.failed = True
                    raise RuntimeError("vLLM actor reply identity differs")
                return message["value"]
            if not self.process.is_alive():
                self.failed = True
                raise RuntimeError(f"vLLM actor exited with code {self.process.exitcode}")

    def _call(self, command: str, **fields):
        if self.process is None or self.failed:
            raise RuntimeError("vLLM actor is not running")
        self.counter += 1
        self.connection.send({"id": self.counter, "command": command, **fields})
        return self._reply(self.counter)

    def start(self) -> dict:
        if self.process is not None:
            raise RuntimeError("the actor starts once")
        ctx = mp.get_context("spawn")
        self.connection, child = ctx.Pipe()
        self.process = ctx.Process(target=_actor_main, args=(child, self.settings), name="tdsv-vllm-actor")
        self.process.start()
        child.close()
        return self._reply(0)

    def generate(self, request: GenerationRequest) -> list[dict]:
        return self._call("generate", request=request)

    def update_head(self, weight: torch.Tensor, version: int) -> dict:
        """Load new LM-head weights (between generations) and check the read-back digest."""
        sent = weight.detach().to("cpu", torch.bfloat16).contiguous()
        expected = tensor_digest(sent)
        receipt = self._call("update_head", weight=sent, version=int(version))
        if receipt["digest"] != expected or receipt["version"] != int(version):
            self.failed = True
            raise RuntimeError(f"vLLM actor loaded a different head: {receipt} (expected {expected})")
        self.head = receipt
        return receipt

    def receipt(self) -> dict:
        return self._call("receipt")

    def close(self) -> dict | None:
        result = None
        if self.process is None:
            return None
        try:
            if self.process.is_alive() and not self.failed:
                result = self._call("close")
        finally:
            self.process.join(timeout=10)
            if self.process.is_alive():  # only this owned child is stopped
                self.process.kill()
                self.process.join()
            self.connection.close()
            self.process = None
        return result


__all__ = ["GenerationRequest", "VLLMActor", "VLLMHeadEngine", "tensor_digest"]
