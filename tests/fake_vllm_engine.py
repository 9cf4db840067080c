"""A stand-in engine for the vLLM actor protocol tests (no vLLM, no GPU): greedy continuation by a
fixed rule and a head kept on the host."""

import torch


class FakeEngine:
    def __init__(self, settings):
        self.head = torch.zeros(4, 3, dtype=torch.bfloat16)
        self.fail_on = settings.get("fail_on")

    def generate(self, request):
        if self.fail_on == "generate":
            raise RuntimeError("engine failure")
        return [{"token_ids": [(p[-1] + i + 1) % 50 for i in range(request.max_tokens)],
                 "log_probs": [-0.5] * request.max_tokens, "finish_reason": "length"} for p in request.prompts]

    def load_head(self, weight):
        from tiny_dsv41_b200.rollout.vllm_actor import tensor_digest

        self.head = weight.clone()
        return [tensor_digest(self.head), tensor_digest(self.head)]  # two workers agree

    def close(self):
        pass
