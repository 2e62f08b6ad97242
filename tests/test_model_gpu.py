"""The drop-in VeraceV1Model (embedding tied to the LM head, ACDE over four decoder layers
with SSSD, CHAM and M-CMoE, final RMSNorm, LM head) against the reference's own
VeraceV1Model.forward (backbone.py:144-210), fp32 on the GPU.

tests/golden/model_golden.npz holds the reference's outputs at a small configuration
(hidden 128, 4 layers, 1 head x 128, D = 128, M-CMoE rank 8 / 8 components): an ACDE
prefill of 2 x 12 tokens (logits, ponder costs, post-norm hidden), two single-token
steps through layer_states (the decode convention of serving/hyper_generate.py:58-77)
and the static-depth path.  Both models hold the same weights through
tests/conftest.py:model_reinit, checked against the reference's fingerprints.
Tolerances: the reference tests' rtol 1e-3 / atol 1e-4 (tests/test_triton_kernels.py:31).
"""
import numpy as np
import pytest
import torch

import verace_v1_b200 as V
from conftest import GOLDEN, model_fingerprints, model_reinit
from gpu_util import to_np

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-3, atol=1e-4)


@pytest.fixture(scope="module")
def case():
    z = np.load(f"{GOLDEN}/model_golden.npz")
    g = {k: z[k] for k in z.files}
    cfg = V.VeraceV1Config(vocab_size=64, hidden_dim=128, num_layers=4, num_heads=1, head_dim=128,
                           spectral_dim=64, chams_holographic_dim=128, mcmoe_rank=8, mcmoe_num_components=8)
    model = V.VeraceV1Model(cfg).eval()
    model_reinit(model, seed=0)
    fps = model_fingerprints(model)
    assert sorted(fps) == sorted(k[3:] for k in g if k.startswith("fp/")), "parameter names differ"
    for k, v in fps.items():
        np.testing.assert_allclose(v, g["fp/" + k], rtol=1e-6, atol=1e-6, err_msg=f"weights of {k} differ")
    return model.cuda(), g


def test_model_prefill_with_acde_matches_reference(case):
    model, g = case
    ids = torch.from_numpy(g["prefill/ids"]).cuda()
    with torch.no_grad():
        logits, depth, hidden = model(ids, return_hidden=True)
    np.testing.assert_allclose(to_np(logits), g["prefill/logits"], **TOL)
    np.testing.assert_allclose(to_np(depth), g["prefill/depth"], **TOL)
    np.testing.assert_allclose(to_np(hidden), g["prefill/hidden"], **TOL)


def test_model_incremental_decode_through_layer_states_matches_reference(case):
    model, g = case
    ids = torch.from_numpy(g["prefill/ids"]).cuda()
    with torch.no_grad():
        _, _, st = model(ids, return_layer_states=True)
        for i in range(2):
            lg, dp, st = model(torch.from_numpy(g[f"step{i}/ids"]).cuda(), layer_states=st, return_layer_states=True)
            np.testing.assert_allclose(to_np(lg), g[f"step{i}/logits"], **TOL)
            np.testing.assert_allclose(to_np(dp), g[f"step{i}/depth"], **TOL)


def test_model_static_depth_matches_reference(case):
    model, g = case
    ids = torch.from_numpy(g["prefill/ids"]).cuda()
    with torch.no_grad():
        lg, dp = model(ids, use_adaptive_depth=False)
    np.testing.assert_allclose(to_np(lg), g["static/logits"], **TOL)
    assert float(dp.min()) == float(dp.max()) == 4.0


def test_model_rejects_images_and_loads_reference_state_dict(case):
    model, _ = case
    with pytest.raises(ValueError, match="outside this path"):
        model(torch.zeros(1, 2, dtype=torch.long, device="cuda"), images=torch.zeros(1, 3, 14, 14, device="cuda"))
    sd = {k: v.clone() for k, v in model.state_dict().items()}
    sd["vision_encoder.patch_embed.weight"] = torch.zeros(1)      # dropped, as out of path
    sd["energy_critic.w_energy.weight"] = torch.zeros(1)
    model.load_reference_state_dict(sd)
