"""The device-side initialisation behind every benchmark number: noise_b200.eggroll.make_params draws EGGROLL's
make_model weights (eggroll.py:38-53 over utils/model.py:149-175) with the same torch calls in the same order. On the
CPU it must equal the oracle's restatement bit for bit, and the oracle's is pinned to the reference's make_model
(tests/test_oracle_golden.py::test_init_matches_reference_make_model). On CUDA the draws come from the CUDA generator
(as the reference's do on CUDA); the GPU test checks the parts that differ from the CPU path: the bf16 round trip of
the embeddings and the c_proj re-draw ranges."""
import pytest
import torch

from oracle import gpt


def test_make_params_cpu_equals_oracle_init_bit_for_bit():
    from noise_b200.eggroll import make_params
    got = make_params('cpu', seed=0)
    want = gpt.init_weights(0, eggroll=True)
    assert list(got) == [n for n, _ in gpt.param_shapes()]
    for name, w in want.items():
        assert got[name].dtype == torch.float32 and torch.equal(got[name], w), name


@pytest.mark.gpu
def test_make_params_cuda_structure():
    from noise_b200.eggroll import make_params
    p = make_params(torch.device('cuda', 0), seed=0)
    for name, t in p.items():
        assert t.is_cuda and t.dtype == torch.float32, name
        if name == 'transformer.wte.weight' or name.startswith('value_embeds.'):
            assert torch.equal(t, t.bfloat16().float()), name  # the CUDA bf16 round trip (model.py:171-175)
        if 'c_proj' in name:
            bound = 1.5 * (3 / t.shape[1]) ** 0.5
            assert t.abs().max().item() <= bound and t.std().item() > 0.5 * bound / 3 ** 0.5, name
    assert torch.equal(p['resid_lambdas'].cpu(), torch.ones(8))
    assert torch.equal(p['x0_lambdas'].cpu(), torch.full((8,), 0.1))
    # the same seed gives the same draws
    again = make_params(torch.device('cuda', 0), seed=0)
    assert all(torch.equal(p[n], again[n]) for n in p)
