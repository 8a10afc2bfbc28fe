"""Generates the golden vectors in this folder from the REFERENCE itself.

Run in a container that has the reference sources (oracle/Makefile compiles
its own src/model/feed_forward.cpp + src/backend/reference/ops.cpp into
oracle/_ref/libref_moe.so):

    python tests/golden/make_golden.py

Each .npz holds the reference's MixtureOfExperts::forward output (renorm off,
no bias: the only semantics the reference has) for seeded synthetic inputs,
plus SHA-256 digests of those inputs so the tests also pin the generator.
`tiny.npz` stores its inputs outright. Configurations without a shared expert
pass the reference a zero shared MLP of width 16, whose output is exactly 0.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402

CASES = {
    # name: (seed, tokens, hidden, experts, top_k, ffn, shared_ffn, bf16_values)
    "c0": (0, 64, 1024, 16, 2, 512, 0, False),
    "c1_layer0_t8": (1, 8, 2048, 64, 6, 1024, 2048, True),
    "tiny": (7, 7, 64, 8, 3, 32, 32, False),
}


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def make_inputs(seed, tokens, hidden, experts, ffn, shared, bf16, layer=0):
    """Inputs in the documented generation order (router, experts' gate/up/down, shared, x)."""
    def g(kind, idx, n, sigma):
        v = O.synth(seed, layer, kind, idx, n, sigma)
        return O.round_bf16(v) if bf16 else v
    H, E, F, S = hidden, experts, ffn, shared
    w = O.MoeWeights(
        router=g(O.KIND_ROUTER, 0, E * H, 0.02).reshape(E, H),
        gate=np.concatenate([g(O.KIND_GATE, e, F * H, 0.02) for e in range(E)]).reshape(E * F, H),
        up=np.concatenate([g(O.KIND_UP, e, F * H, 0.02) for e in range(E)]).reshape(E * F, H),
        down=np.concatenate([g(O.KIND_DOWN, e, H * F, 0.02) for e in range(E)]).reshape(E * H, F),
        shared_gate=(g(O.KIND_SGATE, 0, S * H, 0.02).reshape(S, H) if S else np.zeros((0, H), np.float32)),
        shared_up=(g(O.KIND_SUP, 0, S * H, 0.02).reshape(S, H) if S else np.zeros((0, H), np.float32)),
        shared_down=(g(O.KIND_SDOWN, 0, H * S, 0.02).reshape(H, S) if S else np.zeros((H, 0), np.float32)),
    )
    x = g(O.KIND_X, 0, tokens * H, 1.0).reshape(tokens, H)
    return w, x


def reference_forward(w: O.MoeWeights, x: np.ndarray, top_k: int) -> np.ndarray:
    if w.shared_ffn == 0:  # the reference always has a shared MLP: give it a zero one
        H = w.hidden
        w = O.MoeWeights(w.router, w.gate, w.up, w.down, np.zeros((16, H), np.float32),
                         np.zeros((16, H), np.float32), np.zeros((H, 16), np.float32))
    ref = O.RefMoe(w, top_k)
    try:
        return ref(x)
    finally:
        ref.close()


def main():
    O.build()
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libref_moe.so is missing: the reference sources are needed")
    for name, (seed, T, H, E, K, F, S, bf16) in CASES.items():
        w, x = make_inputs(seed, T, H, E, F, S, bf16)
        y = reference_forward(w, x, K)
        ids = O.moe_forward(w, x, K, renormalize=False).ids  # the oracle's ids; y pins them
        out = dict(seed=seed, tokens=T, hidden=H, experts=E, top_k=K, ffn=F, shared_ffn=S, bf16=bf16, y=y,
                   ids=ids, x_sha=digest(x), router_sha=digest(w.router), gate_sha=digest(w.gate),
                   down_sha=digest(w.down))
        if name == "tiny":
            out.update(x=x, router=w.router, gate=w.gate, up=w.up, down=w.down, shared_gate=w.shared_gate,
                       shared_up=w.shared_up, shared_down=w.shared_down)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print(name, y.shape, float(np.abs(y).max()))


if __name__ == "__main__":
    main()
