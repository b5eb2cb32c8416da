"""The `ab_attention` import name resolves the reference's imports to this build."""
import inspect


def test_reference_import_paths_resolve():
    import ab_attention
    from ab_attention import SamplePlan, ab_attention as layer, apply_plan, build_plan
    from ab_attention import _C, attention, flashinfer_backend

    import ab_attention_b200

    assert ab_attention.__all__ == ["SamplePlan", "ab_attention", "apply_plan", "build_plan"]
    assert build_plan is ab_attention_b200.build_plan and apply_plan is ab_attention_b200.apply_plan
    assert layer is ab_attention_b200.ab_attention and SamplePlan is ab_attention_b200.SamplePlan
    assert attention.build_plan is build_plan  # what the reference's video.py:10 imports
    assert flashinfer_backend.paged_attention is ab_attention_b200.paged_attention
    assert list(inspect.signature(_C.ibcs).parameters) == ["q", "k"]
    assert list(inspect.signature(_C.sip).parameters) == ["scores", "offsets", "ids", "logs"]
    assert list(inspect.signature(build_plan).parameters) == ["q", "k", "sample_pages", "seed", "offsets"]
    assert inspect.signature(build_plan).parameters["sample_pages"].default == 64
    assert inspect.signature(build_plan).parameters["seed"].default == 42


def test_native_stand_in_has_no_cpu_path():
    import pytest
    import torch

    from ab_attention import _C

    q = torch.zeros(1, 1, 256, 128, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        _C.ibcs(q, q)
