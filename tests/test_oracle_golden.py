"""Pins the CPU oracle to the fixtures recorded from the reference (tests/golden)."""
import json
import os

import pytest
import torch

from conftest import GOLDEN
from oracle import paged_plan
from oracle.attention import ContiguousOracle, attend_sequences
from oracle.llama import TinyLlamaOracle, init_params, param_names
from oracle.rope_norm import apply_rotary, rmsnorm, rope_table

ATT = torch.load(os.path.join(GOLDEN, "attention_cases.pt"))
RN = torch.load(os.path.join(GOLDEN, "rope_norm.pt"))
F16 = torch.load(os.path.join(GOLDEN, "fp16_cases.pt"))
ALL_ATT = ATT + F16["attention"]
DTYPES = {"torch.float32": torch.float32, "torch.bfloat16": torch.bfloat16,
          "torch.float16": torch.float16}
with open(os.path.join(GOLDEN, "paged_scenarios.json")) as f:
    SCEN = json.load(f)


@pytest.mark.parametrize("case", ALL_ATT, ids=[c["name"] for c in ALL_ATT])
def test_contiguous_oracle_matches_reference(case):
    dt = DTYPES[case["dtype"]]
    B = len(case["lens"])
    orc = ContiguousOracle(2, B, 128, case["hkv"], case["d"], dt)
    for step in case["steps"]:
        for li, lay in enumerate(step["layers"]):
            out = orc.attend(li, lay["q"], lay["k"], lay["v"], step["start_positions"],
                             step["counts"], step["offsets"])
            exp = lay["out"]
            valid = torch.zeros(exp.shape[:2], dtype=torch.bool)
            for b, (o, n) in enumerate(zip(step["offsets"], step["counts"])):
                valid[b, o:o + n] = True
            torch.testing.assert_close(out[valid], exp[valid], rtol=0, atol=0)


@pytest.mark.parametrize("case", ALL_ATT, ids=[c["name"] for c in ALL_ATT])
def test_per_sequence_formulation_matches_reference(case):
    """attend_sequences (used for large GPU parity cases) against the reference's
    outputs, at the north-star tolerance."""
    dt = DTYPES[case["dtype"]]
    B = len(case["lens"])
    kh = [[torch.zeros(0, case["hkv"], case["d"], dtype=dt) for _ in range(B)] for _ in range(2)]
    vh = [[torch.zeros(0, case["hkv"], case["d"], dtype=dt) for _ in range(B)] for _ in range(2)]
    tol = dict(rtol=1e-4, atol=1e-5) if dt == torch.float32 else dict(rtol=1e-2, atol=2e-2)
    for step in case["steps"]:
        for li, lay in enumerate(step["layers"]):
            qs = []
            for b, (o, n) in enumerate(zip(step["offsets"], step["counts"])):
                kh[li][b] = torch.cat([kh[li][b], lay["k"][b, o:o + n]])
                vh[li][b] = torch.cat([vh[li][b], lay["v"][b, o:o + n]])
                qs.append(lay["q"][b, o:o + n])
            outs = attend_sequences(qs, kh[li], vh[li])
            for b, (o, n) in enumerate(zip(step["offsets"], step["counts"])):
                exp = lay["out"][b, o:o + n].view(n, case["hq"], case["d"])
                torch.testing.assert_close(outs[b], exp, **tol)


def test_rope_tables_match_reference():
    for key in ("t64_1e4", "t128_5e5", "t128_l3"):
        g = RN[f"table_{key}"]
        sc = ({"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
               "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}
              if g["llama3"] else None)
        cos, sin = rope_table(g["dim"], g["max"], g["theta"], sc)
        torch.testing.assert_close(cos[g["rows"]], g["cos"], rtol=0, atol=0)
        torch.testing.assert_close(sin[g["rows"]], g["sin"], rtol=0, atol=0)


def test_product_rope_tables_match_reference():
    """nanoslg_b200.models.precompute_rope_frequencies (vectorised; the tables every GPU
    RoPE launch reads) is bit-exact with the reference's tables, Llama-3 scaling included."""
    from types import SimpleNamespace
    from nanoslg_b200.models import precompute_rope_frequencies
    for key in ("t64_1e4", "t128_5e5", "t128_l3"):
        g = RN[f"table_{key}"]
        sc = ({"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
               "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}
              if g["llama3"] else None)
        cos, sin = precompute_rope_frequencies(g["dim"], g["max"], g["theta"],
                                               SimpleNamespace(rope_scaling=sc))
        assert cos.dtype == torch.float32 and cos.shape == (g["max"], g["dim"])
        torch.testing.assert_close(cos[g["rows"]], g["cos"], rtol=0, atol=0)
        torch.testing.assert_close(sin[g["rows"]], g["sin"], rtol=0, atol=0)


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
def test_rope_and_rmsnorm_match_reference(dt):
    cos, sin = rope_table(128, 4096, 500000.0)
    g = RN[f"rope_{dt}"]
    y = apply_rotary(g["x"], cos[g["pos"]], sin[g["pos"]])
    torch.testing.assert_close(y, g["y"], rtol=0, atol=0)
    g = RN[f"rmsnorm_{dt}"]
    torch.testing.assert_close(rmsnorm(g["x"], g["w"], g["eps"]), g["y"], rtol=0, atol=0)
    g = RN[f"addnorm_{dt}"]
    h = g["x"] + g["r"]
    torch.testing.assert_close(h, g["h"], rtol=0, atol=0)
    torch.testing.assert_close(rmsnorm(h, g["w"], g["eps"]), g["y"], rtol=0, atol=0)


def test_fp16_rope_and_rmsnorm_match_reference():
    cos, sin = rope_table(128, 4096, 500000.0)
    g = F16["rope"]
    y = apply_rotary(g["x"], cos[g["pos"]], sin[g["pos"]])
    torch.testing.assert_close(y, g["y"], rtol=0, atol=0)
    g = F16["rmsnorm"]
    torch.testing.assert_close(rmsnorm(g["x"], g["w"], g["eps"]), g["y"], rtol=0, atol=0)
    g = F16["addnorm"]
    h = g["x"] + g["r"]
    torch.testing.assert_close(h, g["h"], rtol=0, atol=0)
    torch.testing.assert_close(rmsnorm(h, g["w"], g["eps"]), g["y"], rtol=0, atol=0)


def test_plan_restatement_matches_reference():
    n = 0
    for sc in SCEN:
        ps = sc["setup"]["page_size"]
        for rec in sc["records"]:
            if rec["op"][0] != "begin" or "error" in rec:
                continue
            sids, counts = rec["op"][1], rec["op"][2]
            bts = [rec["state"]["block_tables"][s] for s in sids]
            ind, idx, lpl = paged_plan.csr(bts, rec["seq_lens"], ps)
            assert ind == rec["indptr"]
            assert (idx or [0]) == rec["indices"]
            assert (lpl or [0]) == rec["last_page_len"]
            wi = paged_plan.write_targets(bts, rec["start_positions"], counts, ps)
            assert [[list(x) for x in w] for w in wi] == rec["write_info"]
            if not rec["is_decode"]:
                assert paged_plan.qo_indptr(counts) == rec["qo_indptr"]
            n += 1
    assert n > 50


def test_tiny_llama_oracle_greedy_tokens():
    with open(os.path.join(GOLDEN, "tiny_llama.json")) as f:
        g = json.load(f)
    assert g["param_order"] == param_names(g["config"]["num_hidden_layers"])
    torch.set_num_threads(1)
    o = TinyLlamaOracle(g["config"], init_params(g["config"]))
    assert o.greedy(g["prompt"], len(g["tokens"])) == g["tokens"]


def test_tiny_llama_kv8_oracle_greedy_tokens():
    """The batch fixture of the widened tiny model (8/8 heads): each prompt alone through
    the oracle gives the tokens the reference produced for it inside the left-padded
    batch."""
    with open(os.path.join(GOLDEN, "tiny_llama_kv8.json")) as f:
        g = json.load(f)
    assert g["param_order"] == param_names(g["config"]["num_hidden_layers"])
    torch.set_num_threads(1)
    params = init_params(g["config"])
    for prompt, want in zip(g["prompts"], g["tokens"]):
        o = TinyLlamaOracle(g["config"], params)
        assert o.greedy(prompt, len(want)) == want


def test_reference_random_state_dict_matches_oracle_init():
    """models.reference_random_state_dict (the product's copy of the fixtures' init rule)
    gives the oracle's parameters bit for bit, in the reference's parameter order."""
    from types import SimpleNamespace
    from nanoslg_b200.models import reference_random_state_dict
    for name in ("tiny_llama.json", "tiny_llama_kv8.json"):
        with open(os.path.join(GOLDEN, name)) as f:
            g = json.load(f)
        got = reference_random_state_dict(SimpleNamespace(**g["config"]))
        want = init_params(g["config"])
        assert list(got) == g["param_order"]
        for k in want:
            assert torch.equal(got[k], want[k]), k
