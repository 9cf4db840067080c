"""GRPO / Token-TIS objectives and response scoring against the reference implementation."""

import pytest
import torch

from tiny_dsv41_b200.rl import algorithm as A

from ref_oracle import import_reference, reference_available

pytestmark = pytest.mark.skipif(not reference_available(), reason="reference not installed under baseline/_ref")


def _inputs(seed=0):
    g = torch.Generator().manual_seed(seed)
    lengths = [3, 5, 1, 4]
    pol = [(-torch.rand(n, generator=g) * 3).requires_grad_() for n in lengths]
    beh = [p.detach() + 0.1 * torch.randn(p.shape, generator=g) for p in pol]
    beh = [b.clamp(max=0) for b in beh]
    ref = [p.detach() - 0.05 * torch.rand(p.shape, generator=g) for p in pol]
    old = [p.detach() + 0.05 * torch.randn(p.shape, generator=g) for p in pol]
    old = [o.clamp(max=0) for o in old]
    adv = torch.randn(len(lengths), generator=g)
    return pol, beh, ref, old, adv


def test_grpo_and_token_tis_match_reference():
    import_reference()
    from dsv41_train.rl import algorithm as R

    for kl in (0.0, 0.05):
        pol, beh, ref, _, adv = _inputs(1)
        loss, stats = A.grpo_loss(pol, beh, adv, 0.2, ref, kl)
        loss.backward()
        grads = [p.grad.clone() for p in pol]
        pol2 = [p.detach().clone().requires_grad_() for p in pol]
        loss2, stats2 = R.grpo_loss(pol2, beh, adv, 0.2, ref, kl)
        loss2.backward()
        assert torch.allclose(loss, loss2) and stats.keys() == stats2.keys()
        assert all(torch.allclose(a, b.grad) for a, b in zip(grads, pol2))
    pol, beh, _, old, adv = _inputs(2)
    loss, stats = A.decoupled_token_tis_loss(pol, old, beh, adv, 0.2, 2.0)
    loss2, stats2 = R.decoupled_token_tis_loss([p.detach().clone().requires_grad_() for p in pol], old, beh, adv, 0.2, 2.0)
    assert torch.allclose(loss, loss2)
    assert stats.keys() == stats2.keys()
    for k in stats:
        assert abs(stats[k] - stats2[k]) < 1e-6 * max(1.0, abs(stats2[k])), k
    rewards = [0.0, 1.0, 1.0, 0.5]
    assert torch.allclose(A.group_advantages(rewards), R.group_advantages(rewards))


def test_response_log_probs_dsv4_matches_reference():
    import_reference()
    from dsv41_train.models.dsv4.config import DeepSeekV41Config as RC
    from dsv41_train.models.dsv4.model import DeepSeekV41ForCausalLM as RM
    from dsv41_train.rl import algorithm as R

    from tiny_dsv41_b200.models.dsv4 import DeepSeekV41Config, DeepSeekV41ForCausalLM

    torch.manual_seed(0)
    mine = DeepSeekV41ForCausalLM(DeepSeekV41Config.tiny())
    ref = RM(RC.tiny())
    ref.load_state_dict(mine.state_dict())
    prompts, responses = [[1, 4, 5], [1, 9, 6, 7]], [[7, 8, 2], [10, 2]]
    a = A.response_log_probs_batch(mine, prompts, responses, 0.8)
    b = R.response_log_probs_batch(ref, prompts, responses, 0.8)
    assert all(torch.allclose(x, y, atol=1e-5) for x, y in zip(a, b))


def test_gsm8k_selection_and_metrics(tmp_path):
    from pathlib import Path

    from tiny_dsv41_b200.rl.gsm8k import formatting_correct, select_records, wilson_interval
    from tiny_dsv41_b200.rl.tokenizer import ModelTokenizer

    tok = ModelTokenizer(Path(__file__).resolve().parents[1] / "examples" / "tiny-dsv41")
    rows = [{"id": f"gsm8k:train:{i}", "question": "what is the sum of 1 and " + "2 " * i, "answer": "3"}
            for i in range(6)]
    selected, excluded = select_records(rows, rows[:3], tok, max_prompt_tokens=27, max_train_groups=2,
                                        eval_questions=1)
    assert len(selected["train"]) == 2 and all(len(r.prompt_ids) <= 27 for r in selected["train"])
    assert len(excluded["train"]) + 2 <= len(rows)
    assert formatting_correct("so #### 42") and not formatting_correct("42")
    low, high = wilson_interval(5, 10)
    assert 0.23 < low < 0.24 and 0.76 < high < 0.77


def test_learner_batch_planner_matches_reference():
    import random

    from tests.ref_oracle import import_reference, reference_available
    from tiny_dsv41_b200.rl import learner_batch_planner as P

    cells = P.parse_learner_batch_shapes("4:512,8:256,2:2047")
    rng = random.Random(0)
    lengths = [rng.randrange(1, 2048) for _ in range(32)]
    plan = P.plan_learner_microbatches(lengths, 4, cells)
    covered = sorted(i for b in plan for i in b["response_indices"])
    assert covered == list(range(32))
    own = [P.plan_response_ownership(lengths, r, 3) for r in range(3)]
    assert len({len(o) for o in own}) == 1
    if reference_available():
        import_reference()
        from dsv41_train.rl import learner_batch_planner as R

        assert R.parse_learner_batch_shapes("4:512,8:256,2:2047") == cells
        assert R.plan_learner_microbatches(lengths, 4, cells) == plan
        assert [R.plan_response_ownership(lengths, r, 3) for r in range(3)] == own
