"""On-device calibration on the GPU: the bisection run as device tensor code
(calibrate_from_qk, one read-back) picks the value the reference's host loop
picks over the same GPU lag scores (corr_mask_fraction at each step).  The file
sorts after the kernel tests, so under -x they run first."""
import pytest
import torch

from fftsparse_b200.params import derive_mask_params
from fftsparse_b200.prefill import corr_mask_fraction
from oracle.synth import make_inputs
from tests.test_calibrate import KW, reference_bisection

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,target", [("topk", 0.05), ("threshold", 0.1)])
def test_gpu_calibration_equals_reference_loop(mode, target):
    import fftsparse_b200 as F
    from fftsparse_b200.calibrate import calibrate_from_qk
    F.load_library()
    layers = []
    for seed in (0, 1):
        q, k, _ = make_inputs(8192, num_q_heads=4, num_kv_heads=2, dtype=torch.bfloat16, expand=False, seed=seed)
        layers.append((q.cuda(), k.cuda()))
    topk = mode == "topk"
    masks = [F.fft_block_mask(q, k, correlation_selection_mode=mode, correlation_topk_ratio=0.0 if topk else 0.2,
                              **KW) for q, k in layers]

    def fraction_of(val):
        fr = []
        for (q, k), m in zip(layers, masks):
            p = derive_mask_params(q.shape[2], block_size=128, correlation_selection_mode=mode,
                                   correlation_topk_ratio=val if topk else 0.2,
                                   corr_threshold=1.0 if topk else val, **KW)
            if p.corr_on:
                fr.append(corr_mask_fraction(m.corr, p))
        return sum(fr) / len(fr)

    best, corr_ret, final_ret = calibrate_from_qk(layers, target, correlation_selection_mode=mode, **KW)
    assert best == reference_bisection(fraction_of, target, topk)
    assert abs(corr_ret - target) < 0.01
    assert 0.0 < final_ret <= 1.0
