"""Plan-reuse schedule (ab_attention/video.py:53-87): anchors, seeds, dense steps.

The CPU tests drive the schedule with build/apply stand-ins; the GPU test runs
real plans and checks reuse against a fresh build with the anchor's seed."""
import pytest
import torch

from ab_attention_b200 import video


def test_anchor_and_seed_follow_the_reference_schedule():
    anchors = [video.anchor_step(s) for s in range(11, 51)]
    assert anchors[:8] == [11, 11, 11, 11, 15, 15, 15, 15]
    assert sorted(set(anchors)) == list(range(11, 51, 4))
    assert video.plan_seed(3, 15) == 42 + 3 * 1_000_003 + 15 * 97


def test_dense_steps_and_layer_zero(monkeypatch):
    sched = video.VideoAttention(64)
    assert not sched.is_sparse(1)            # step 1
    sched.step_end(None, 9, None, {})         # -> step 11
    assert sched.step == 11 and sched.is_sparse(1) and not sched.is_sparse(0)
    assert not video.VideoAttention(64, dense=True).is_sparse(5)


def test_plans_built_on_anchors_and_reused_between(monkeypatch):
    built = []

    def fake_build(q, k, *, sample_pages, seed):
        built.append(seed)
        return video.SamplePlan(torch.full((2, 1, 32), seed), torch.zeros(2, 1, 32))

    applied = []
    monkeypatch.setattr(video, "build_plan", fake_build)
    monkeypatch.setattr(video, "apply_plan", lambda q, k, v, plan, **kw: applied.append(int(plan[0][0, 0, 0])))
    sched = video.VideoAttention(1)
    x = torch.zeros(1)
    for step in range(11, 20):
        sched.step = step
        sched.attend(2, x, x, x)
    assert built == [video.plan_seed(2, 11), video.plan_seed(2, 15), video.plan_seed(2, 19)]
    assert applied == [video.plan_seed(2, 11)] * 4 + [video.plan_seed(2, 15)] * 4 + [video.plan_seed(2, 19)]


@pytest.mark.gpu
def test_reused_plan_equals_anchor_plan_on_gpu():
    from ab_attention_b200 import apply_plan, build_plan
    from ab_attention_b200.synthetic import smooth_field

    q, k, v = (t.unsqueeze(0) for t in smooth_field(2, 4, 16, 32, seed=5, device="cuda"))
    sched = video.VideoAttention(2)
    sched.step = 13
    o13 = sched.attend(1, q, k, v)
    sched.step = 14                              # same anchor (11): stored plan reused
    o14 = sched.attend(1, q, k, v)
    want = apply_plan(q, k, v, build_plan(q, k, sample_pages=2, seed=video.plan_seed(1, 11)))
    assert torch.equal(o13, want) and torch.equal(o14, want)
    host = video.VideoAttention(2, host_plans=True)
    host.step = 12
    host.attend(1, q, k, v)
    host.step = 13
    assert torch.equal(host.attend(1, q, k, v), want)
    assert host.plans[1][1].descriptor.device.type == "cpu"
