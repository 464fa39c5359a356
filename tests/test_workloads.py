"""The seeded input generator: determinism, quantisation layout and value
ranges, and the routing variants the benchmark configurations use."""
from __future__ import annotations

import torch

import moe_oracle
import workloads


def test_deterministic_and_seed_sensitive():
    a = workloads.make_routing_inputs(8, 3)
    b = workloads.make_routing_inputs(8, 3)
    c = workloads.make_routing_inputs(8, 4)
    assert torch.equal(a["routing_logits"], b["routing_logits"])
    assert torch.equal(a["routing_bias"].float(), b["routing_bias"].float())
    assert not torch.equal(a["routing_logits"], c["routing_logits"])


def test_row_quantisation_round_trip():
    x = torch.randn(5, 7168)
    q, s = workloads.quantize_rows_1x128(x)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (56, 5)
    deq = moe_oracle.dequant_hidden(q, s)
    blk = x.view(5, 56, 128).abs().amax(dim=2)
    assert torch.allclose(s.t(), blk / 448.0)
    # e4m3 keeps 3 mantissa bits: relative error <= 2^-4 of the block max
    assert float(((deq - x).abs().view(5, 56, 128) / blk.unsqueeze(2)).max()) <= 2.0 ** -4 + 1e-6
    assert float(q.float().abs().max()) <= 448.0


def test_block_quantisation_round_trip():
    w = torch.randn(256, 384) * 0.02
    q, s = workloads.quantize_blocks_128x128(w)
    assert s.shape == (2, 3)
    deq = moe_oracle.dequant_block(q, s)
    blk = w.view(2, 128, 3, 128).abs().amax(dim=(1, 3))
    err = (deq - w).abs().view(2, 128, 3, 128).amax(dim=(1, 3))
    assert bool((err <= blk * 2.0 ** -4 + 1e-9).all())


def test_expert_subset_matches_full_generation():
    full = workloads.make_expert_weights(7, 5)
    again = workloads.make_expert_weights(7, 5)
    for a, b in zip(full, again):
        assert torch.equal(a.float(), b.float())
    other = workloads.make_expert_weights(7, 6)
    assert not torch.equal(full[0].float(), other[0].float())


def test_hot_variant_routes_most_tokens_to_the_hot_experts():
    r = workloads.make_routing_inputs(1024, 0, "cpu", "hot")
    idx, _ = moe_oracle.route(r["routing_logits"], r["routing_bias"], 2.5)
    for le in workloads.HOT_LOCAL_EXPERTS:
        assert float((idx == le).any(dim=1).float().mean()) > 0.9


def test_zipf_variant_is_skewed():
    r = workloads.make_routing_inputs(4096, 0, "cpu", "zipf")
    idx, _ = moe_oracle.route(r["routing_logits"], r["routing_bias"], 2.5)
    counts = torch.bincount(idx.flatten(), minlength=256).sort(descending=True).values
    assert int(counts[:16].sum()) > 4 * int(counts[-128:].sum())


def test_weight_seed_separates_shards():
    a = workloads.make_inputs(2, 1, experts=[0], weight_seed=10)
    b = workloads.make_inputs(2, 1, experts=[0], weight_seed=11)
    assert torch.equal(a["routing_logits"], b["routing_logits"])
    assert not torch.equal(a["gemm1_weights"][0].float(), b["gemm1_weights"][0].float())
