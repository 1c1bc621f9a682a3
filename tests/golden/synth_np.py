"""Config-1 inputs of the golden fixtures, from the seeded numpy generator in
oracle/synth.py (test infrastructure)."""
import os
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", ".."))
from oracle.synth import digest, rope_np, synth_kv, synth_q  # noqa: E402,F401

# Config 1 of the benchmark plan: batch 2 at T = 1000 and at T = 777, 8 q / 2 kv heads.
CONFIG1 = [dict(name=f"config1_T{T}", B=2, T=T, Hq=8, Hkv=2, theta=1e6, seed_k=100 + T, seed_v=200 + T,
                seed_q=300 + T) for T in (1000, 777)]


def config1_inputs(case):
    TS = -(-case["T"] // 16) * 16
    k = synth_kv(case["seed_k"], case["B"], TS, case["Hkv"], theta=case["theta"], key=True)
    v = synth_kv(case["seed_v"], case["B"], TS, case["Hkv"], theta=case["theta"], key=False)
    q = synth_q(case["seed_q"], case["B"], case["Hq"])
    return q, k, v
