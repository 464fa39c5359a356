"""Properties of the routing and permutation restatement itself (the
reference's rules: top-2 group sums, top-4 groups, top-8 experts, weights
from unbiased scores renormalised and scaled, ties to the lower index)."""
from __future__ import annotations

import torch

import moe_oracle
import workloads


def test_routing_rules_hold():
    r = workloads.make_routing_inputs(512, 3)
    idx, w = moe_oracle.route(r["routing_logits"], r["routing_bias"], 2.5)
    assert idx.shape == (512, 8) and w.shape == (512, 8)
    # distinct experts, from at most 4 groups
    assert bool((idx.sort(dim=1).values.diff(dim=1) > 0).all())
    groups = idx // 32
    assert max(len(set(g.tolist())) for g in groups) <= 4
    # weights renormalised and scaled
    torch.testing.assert_close(w.sum(dim=1), torch.full((512,), 2.5), rtol=1e-5, atol=0)
    # best first by biased score
    s = torch.sigmoid(r["routing_logits"]) + r["routing_bias"].float()
    sel = s.gather(1, idx)
    assert bool((sel.diff(dim=1) <= 0).all())


def test_group_choice_uses_top2_sum():
    # one huge expert in group 0 but the rest of group 0 low: the top-2 sum,
    # not the max, decides the group
    logits = torch.full((1, 256), -4.0)
    logits[0, 5] = 8.0                              # group 0: one high expert
    for g in range(1, 5):
        logits[0, 32 * g: 32 * g + 2] = 2.0         # groups 1-4: two good experts each
    bias = torch.zeros(256)
    idx, _ = moe_oracle.route(logits, bias, 1.0)
    chosen_groups = set((idx[0] // 32).tolist())
    assert chosen_groups == {1, 2, 3, 4}


def test_ties_break_to_lower_index():
    logits = torch.zeros(1, 256)
    idx, w = moe_oracle.route(logits, torch.zeros(256), 1.0)
    assert idx[0].tolist() == list(range(8))        # groups 0-3 kept, experts 0-7 chosen
    torch.testing.assert_close(w[0], torch.full((8,), 1 / 8))


def test_permutation_segments():
    r = workloads.make_routing_inputs(300, 5)
    idx, w = moe_oracle.route(r["routing_logits"], r["routing_bias"], 2.5)
    for off in (0, 32, 224, 256, -32):
        seg, tok, pw = moe_oracle.permute(idx, w, off)
        assert seg[0] == 0 and bool((seg.diff() >= 0).all()) and int(seg[-1]) == tok.numel()
        local = (idx >= off) & (idx < off + 32)
        assert tok.numel() == int(local.sum())
        for e in range(32):
            t = tok[seg[e]:seg[e + 1]]
            assert bool((t.diff() > 0).all())               # ascending, no duplicates
            assert bool((idx[t] == off + e).any(dim=1).all())


def test_token_subset_matches_full_rows():
    inp = workloads.make_inputs(6, 2, experts=None)
    full = moe_oracle.moe_forward(*workloads.as_args(inp), return_fp32=True)
    sub = torch.tensor([1, 4])
    part = moe_oracle.moe_forward(*workloads.as_args(inp), token_subset=sub, return_fp32=True)
    torch.testing.assert_close(part, full[sub], rtol=1e-6, atol=1e-6)


def test_output_close_metric():
    ref = torch.tensor([[1.0, -2.0, 0.5, 0.0]])
    ok, matched, _, ref_max = moe_oracle.output_close(ref + 0.01, ref)
    assert ok and matched == 1.0 and ref_max == 2.0
    bad = ref.clone()
    bad[0, 0] += 1.0
    ok, matched, _, _ = moe_oracle.output_close(bad, ref)
    assert not ok and matched == 0.75
