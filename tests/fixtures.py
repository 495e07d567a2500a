"""Load golden fixtures (written by tests/golden/make_golden.py from the reference) and
rebuild the seeded weights they were made with."""
from __future__ import annotations

from pathlib import Path

import numpy as np

import synth
from oracle.moe_oracle import MoEParams

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str):
    return dict(np.load(GOLDEN / f"{name}.npz"))


def std_linear(name: str):
    """StandardMoE linear fixture -> (fixture dict, MoEParams with x@W expert layout)."""
    f = load(name)
    E, d, M, seed, fp16 = [int(v) for v in f["meta"]]
    g = synth.normal(seed, (E, d), 0.02)
    W = synth.normal(seed + 1, (E, d, d), 0.02)           # nn.Linear weight [out, in]
    p = MoEParams(gate=g, expert_type="linear", expert_w=np.ascontiguousarray(W.transpose(0, 2, 1)))
    f.update(E=E, d=d, M=M, fp16=bool(fp16), expert_lin=W)
    return f, p


def std_swiglu(name: str):
    f = load(name)
    E, d, F, M, seed, _ = [int(v) for v in f["meta"]]
    w1, w3, w2 = synth.swiglu_weights(seed, E, d, F, init="xavier")
    g = synth.xavier_normal(seed + 5, (E, d))
    p = MoEParams(gate=g, expert_type="swiglu", w1=w1, w3=w3, w2=w2)
    f.update(E=E, d=d, F=F, M=M)
    return f, p


def ult_linear(name: str):
    f = load(name)
    E, d, M, seed, ws = [int(v) for v in f["meta"]]
    g = synth.normal(seed, (E, d), 0.02)
    W = synth.normal(seed + 1, (E, d, d), 0.02)           # x @ W layout
    p = MoEParams(gate=g, expert_type="linear", expert_w=W)
    f.update(E=E, d=d, M=M, ws=ws)
    return f, p


STD_LINEAR = ["std_linear_fp32_E8_d64_M37", "std_linear_fp32_E16_d128_M1",
              "std_linear_fp32_E8_d64_M0", "std_linear_fp32_E64_d256_M300"]
STD_SWIGLU = ["std_swiglu_fp32_E4_d32_F64_M29", "std_swiglu_fp32_E8_d128_F256_M70",
              "std_swiglu_fp32_E8_d512_F2048_M8", "std_swiglu_fp32_E8_d512_F2048_M64"]
ULT_LINEAR = ["ult_linear_fp32_ws1_E8_d64_M50", "ult_linear_fp32_ws2_E8_d32_M23",
              "ult_linear_fp32_ws4_E8_d32_M17"]


def std_swiglu_lowp(name: str):
    """16-bit reference run: weights are synth.swiglu_weights(seed, init='normal')."""
    f = load(name)
    E, d, F, M, seed = [int(v) for v in f["meta"]]
    w1, w3, w2 = synth.swiglu_weights(seed, E, d, F, init="normal", std=0.02)
    g = synth.normal(seed + 5, (E, d), 0.02)
    p = MoEParams(gate=g, expert_type="swiglu", w1=w1, w3=w3, w2=w2)
    f.update(E=E, d=d, F=F, M=M)
    return f, p


GRADS = ["grad_std_linear_fp32_E8_d48_M41", "grad_std_swiglu_fp32_E4_d32_F64_M29",
         "grad_std_swiglu_fp32_E8_d32_F48_M57"]


def std_grads(name: str):
    """Reference StandardMoE gradients (autograd through its forward, fp32)."""
    f = load(name)
    E, d, F, M, seed, swiglu = [int(v) for v in f["meta"]]
    if swiglu:
        w1, w3, w2 = synth.swiglu_weights(seed, E, d, F, init="xavier")
        p = MoEParams(gate=synth.xavier_normal(seed + 5, (E, d)), expert_type="swiglu", w1=w1, w3=w3, w2=w2)
    else:
        W = synth.normal(seed + 1, (E, d, d), 0.02)       # nn.Linear weight [out, in]
        p = MoEParams(gate=synth.normal(seed, (E, d), 0.02), expert_type="linear",
                      expert_w=np.ascontiguousarray(W.transpose(0, 2, 1)))
    f.update(E=E, d=d, F=F, M=M)
    return f, p
