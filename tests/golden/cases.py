"""Golden-fixture cases and their seeded inputs (shared by make_golden.py and the tests).

Shapes mirror the reference's own parity tests (tests/test_attnres_ops.py:884-1030)
and BASELINE config 1 (base AttnRes, S=5, N=2x128, d=256, fp32, query ~ N(0, 0.02)).
Inputs come from numpy's PCG64 generator with a fixed seed per case.
"""
import numpy as np

CASES = [
    # LRID static query, mirrors test_fused_lrid_static_query_matches_torch (:898-913)
    dict(name="lrid_static_h1_nokn", kind="lrid", S=6, B=2, T=7, D=128, R=32, H=1, scale=0.25,
         key_norm=False, query="static", seed=11),
    dict(name="lrid_static_h1_kn", kind="lrid", S=6, B=2, T=7, D=128, R=32, H=1, scale=0.25,
         key_norm=True, query="static", seed=12),
    dict(name="lrid_static_h4_kn", kind="lrid", S=6, B=2, T=7, D=128, R=32, H=4, scale=0.25,
         key_norm=True, query="static", seed=13),
    dict(name="lrid_static_h4_nokn", kind="lrid", S=6, B=2, T=7, D=128, R=32, H=4, scale=0.25,
         key_norm=False, query="static", seed=14),
    # dynamic query, mirrors test_fused_lrid_dynamic_query_matches_torch (:975-989)
    dict(name="lrid_dynamic_h2", kind="lrid", S=4, B=2, T=6, D=128, R=32, H=2, scale=0.5,
         key_norm=True, query="dynamic", seed=15),
    # gated hybrid query q = q_static + gate * q_dynamic (model.py:2104-2110), BASELINE config 3 shape family
    dict(name="lrid_gated_h4", kind="lrid", S=5, B=2, T=5, D=64, R=32, H=4, scale=0.35,
         key_norm=True, query="gated", seed=16),
    # output norm (H=1: fused per-head norm; H=2: full-row _norm of the output)
    dict(name="lrid_outnorm_h1", kind="lrid", S=5, B=1, T=8, D=64, R=16, H=1, scale=0.125,
         key_norm=True, query="static", normalize_output=True, seed=17),
    dict(name="lrid_outnorm_h2", kind="lrid", S=5, B=1, T=8, D=64, R=16, H=2, scale=0.125,
         key_norm=True, query="static", normalize_output=True, seed=18),
    # learned per-source logit biases (count-prior route, attnres_ops.py:4259-4315)
    dict(name="lrid_bias_h2", kind="lrid", S=4, B=2, T=3, D=32, R=16, H=2, scale=0.5,
         key_norm=True, query="static", bias=True, seed=19),
    # rank-512 single head (test_fused_lrid_r512_single_head_eval_matches_torch, :916-931)
    dict(name="lrid_r512_h1", kind="lrid", S=3, B=1, T=3, D=1024, R=512, H=1, scale=1.0,
         key_norm=True, query="static", seed=26),
    # keys projected from the values (lrid_key_from_value, model.py:344-356)
    dict(name="lrid_kv_h2", kind="lrid_kv", S=5, B=2, T=5, D=128, R=32, H=2, scale=0.5,
         key_norm=True, query="static", seed=31),
    dict(name="lrid_kv_h1_nonorm", kind="lrid_kv", S=4, B=1, T=6, D=64, R=16, H=1, scale=0.25,
         key_norm=True, query="static", value_norm=False, seed=32),
    # cached-logit block read (attention_residual_phase1_from_logits, attnres_ops.py:3910)
    dict(name="phase1_q3", kind="phase1", S=5, Q=3, B=2, T=6, D=64, seed=41),
    dict(name="phase1_q2_norm", kind="phase1", S=4, Q=2, B=1, T=9, D=32, normalize_output=True, seed=42),
    # cached-logit phase 2: merge of the live partial block (attnres_ops.py:3964-4160)
    dict(name="phase2_lrid", kind="phase2", mode="lrid", S=1, B=2, T=7, D=48, R=16, scale=0.25, key_norm=True,
         seed=51),
    dict(name="phase2_lrid_bias_norm", kind="phase2", mode="lrid", S=1, B=1, T=9, D=64, R=32, scale=0.5,
         key_norm=False, bias=True, normalize_output=True, seed=52),
    dict(name="phase2_base", kind="phase2", mode="base", S=1, B=2, T=5, D=32, key_norm=True, seed=53),
    dict(name="phase2_base_bias_raw", kind="phase2", mode="base", S=1, B=1, T=8, D=40, key_norm=False, bias=True,
         query_std=0.1, seed=54),
    dict(name="phase2_logit_norm", kind="phase2", mode="logit", S=1, B=2, T=6, D=24, normalize_output=True,
         seed=55),
    # base AttnRes read, mirrors test_fused_base_attnres_matches_torch (:884-895)
    dict(name="base_small_kn", kind="base", S=5, B=2, T=5, D=64, key_norm=True, seed=21),
    dict(name="base_small_nokn", kind="base", S=5, B=2, T=5, D=64, key_norm=False, seed=22),
    dict(name="base_outnorm_bias", kind="base", S=4, B=1, T=6, D=32, key_norm=True,
         normalize_output=True, bias=True, seed=23),
    # S=5, N=2x128, d=256, fp32, static query ~ N(0, 0.02)
    dict(name="base_config1", kind="base", S=5, B=2, T=128, D=256, key_norm=True, seed=1,
         query_std=0.02, keep_tokens=16),
]


def case_inputs(case):
    rng = np.random.default_rng(case["seed"])
    S, N, D = case["S"], case["B"] * case["T"], case["D"]
    f = lambda *shape: rng.standard_normal(shape).astype(np.float32)  # noqa: E731
    inp = {"values": f(S, N, D)}
    if case["kind"] in ("lrid", "lrid_kv"):
        H, R = case["H"], case["R"]
        inp["keys"] = f(S, N, R)
        inp["query"] = f(H, R // H)
        inp["query_dynamic"] = f(N, H, R // H)
        inp["gate"] = (0.1 + 0.2 * rng.standard_normal(H)).astype(np.float32)
    elif case["kind"] == "phase2":
        inp = {"partial_value": f(N, D), "interblock_output": f(N, D), "interblock_lse": f(N),
               "grad_output": f(N, D), "logit_bias": np.float32(rng.standard_normal())}
        if case["mode"] == "lrid":
            inp["partial_key"] = f(N, case["R"])
            inp["query"] = f(case["R"])
        elif case["mode"] == "base":
            inp["query"] = (f(D) * np.float32(case.get("query_std", 1.0))).astype(np.float32)
        else:
            inp["partial_logit"] = f(N)
        return inp
    elif case["kind"] == "phase1":
        inp["logits"] = f(case["Q"], S, N)
        inp["grad_lse"] = f(case["Q"], N)
        inp["grad_output"] = f(case["Q"], N, D)
        return inp
    else:
        inp["query"] = (f(D) * np.float32(case.get("query_std", 1.0))).astype(np.float32)
    if case["kind"] == "lrid_kv":
        inp["key_weight"] = (rng.standard_normal((case["R"], D)) / np.sqrt(D)).astype(np.float32)
    inp["logit_bias"] = rng.standard_normal(S).astype(np.float32)
    inp["grad_output"] = f(N, D)
    return inp
