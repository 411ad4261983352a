"""The reference module's own self-test suite (KeSSieKernelTests,
kessie_hip_kernels.py:613-747), mirrored in kessie_b200.kessie_hip_kernels:
on CPU every test skips and passes, as the reference's does without Triton;
on a GPU every test passes on this library's kernels at the reference's
thresholds."""

import pytest
import torch


def test_selftest_suite_skips_without_gpu():
    from kessie_b200 import kessie_hip_kernels as K
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    t = K.KeSSieKernelTests("cpu")
    assert t.run_all() is True
    assert t.bench_fused_vs_separate(256) is None


@pytest.mark.gpu
def test_selftest_suite_passes_on_gpu():
    from kessie_b200 import kessie_hip_kernels as K
    torch.manual_seed(0)
    t = K.KeSSieKernelTests("cuda")
    assert t.test_windowed_attention_correctness()
    assert t.test_fused_fog_attention()
    assert t.test_rope_remap()
    assert t.test_paged_kv_cache()
    t_sep, t_fused = t.bench_fused_vs_separate(1024)
    assert t_sep > 0 and t_fused > 0
