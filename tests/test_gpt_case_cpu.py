"""Host-side pieces of the data-parallel GPT driver (no GPU): the model has
the parameter count of the benchmark configuration, per-rank data streams
differ, and the FLOP count follows 6 * params * tokens plus attention."""
import torch

from cuda_transformer_b200 import gpt_case


def test_default_model_size():
    m = gpt_case.GPT()  # 6 x 384, 6 heads, ctx 256, vocab 65, tied lm_head
    n = gpt_case.n_params(m)
    assert n == 6 * 1_774_464 + 65 * 384 + 256 * 384 + 2 * 384 + 65


def test_rank_batches_are_seeded_per_rank():
    a = gpt_case.rank_batches(1000, 2, 4, 16, 65)
    b = gpt_case.rank_batches(1001, 2, 4, 16, 65)
    a2 = gpt_case.rank_batches(1000, 2, 4, 16, 65)
    assert torch.equal(a[0][0], a2[0][0]) and not torch.equal(a[0][0], b[0][0])
    x, y = a[0]
    assert x.shape == (4, 16) and torch.equal(x[:, 1:], y[:, :-1])
    assert int(x.max()) < 65 and int(x.min()) >= 0


def test_step_flops():
    f = gpt_case.step_flops(1000, 2, 8, 16, 10)
    assert f == 6.0 * 1000 * 10 + 3.0 * 2.0 * 2 * 16 * 8 * 10
