"""Generate the golden fixtures in tests/golden/ from the CPU oracle.

    python tests/golden/make_golden.py

The reference (Metal kernels run through MLX/MTPLX) cannot execute here, so
these vectors are produced by the oracle (oracle/), whose format and mask
rules are pinned against the reference's own known-answer test and code in
tests/test_oracle.py. The fixtures freeze small seeded cases, so that the GPU
parity tests and the oracle are compared against the same committed bytes.
Seeds: 2000 + case index.
"""

from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import attention, bf16, gen, kv, qmm, tree  # noqa: E402

QMM_CASES = [  # (M, N, K) small shapes incl. odd M and K not a multiple of 512
    (1, 128, 128),
    (3, 128, 256),
    (8, 256, 512),
    (16, 128, 640),
    (33, 256, 192),
    (64, 128, 1024),
    (100, 128, 320),
]

ATTN_CASES = [  # (B, Hq, Hkv, T, n_kv, cap, fmt, mode)
    (1, 6, 1, 3, 70, 96, "bf16", "parents"),
    (1, 24, 4, 8, 300, 320, "bf16", "parents"),
    (2, 12, 2, 16, 200, 256, "ref_q8", "parents"),
    (1, 6, 1, 32, 777, 800, "mlx_q8", "parents"),
    (2, 4, 2, 5, 130, 160, "bf16", "bits_tail"),
    (1, 8, 4, 1, 65, 96, "ref_q8", "parents"),
]


def qmm_fixture(i, m, n, k):
    rng = np.random.default_rng(2000 + i)
    x = gen.x_bf16(rng, m, k)
    wq, s, b = gen.weights_w4g64(rng, n, k)
    y = qmm.qmm(x, wq, s, b)
    deq = qmm.dequantize(wq, s, b)
    return dict(x=x, w=wq, scales=s, biases=b, y=y.astype(np.float32), deq=deq)


def attn_fixture(i, bsz, hq, hkv, t, n_kv, cap, fmt, mode):
    rng = np.random.default_rng(3000 + i)
    d = 256
    q = bf16.f32_to_bf16_bits(rng.standard_normal((bsz, hq, t, d), dtype=np.float32))
    kf = rng.standard_normal((bsz, hkv, cap, d), dtype=np.float32)
    vf = rng.standard_normal((bsz, hkv, cap, d), dtype=np.float32)
    out = dict(q=q, n_kv=np.int64(n_kv), fmt=np.array(fmt))
    if fmt == "bf16":
        kb, vb = bf16.f32_to_bf16_bits(kf), bf16.f32_to_bf16_bits(vf)
        out.update(k=kb, v=vb)
        kval, vval = bf16.bf16_bits_to_f32(kb), bf16.bf16_bits_to_f32(vb)
    elif fmt == "ref_q8":
        kq, ks = kv.quantize_rows(kf)
        vq, vs = kv.quantize_rows(vf)
        out.update(k=kq, v=vq, k_scale=ks, v_scale=vs)
        kval, vval = kv.dequant_rows(kq, ks), kv.dequant_rows(vq, vs)
    else:
        kw, kss, kbb = kv.quantize_g64(kf)
        vw, vss, vbb = kv.quantize_g64(vf)
        out.update(k=kw, v=vw, k_scales=kss, k_biases=kbb, v_scales=vss, v_biases=vbb)
        kval, vval = kv.dequant_g64(kw, kss, kbb), kv.dequant_g64(vw, vss, vbb)
    parents = np.stack([gen.tree_parents(rng, t) for _ in range(bsz)])
    if mode == "parents":
        bits = np.stack([tree.ancestor_bits_u64(p) for p in parents])
        tail = t
    else:  # explicit masks over a tail longer than the query count
        tail = t + 3
        bits = rng.integers(0, 2**tail, size=(bsz, t), dtype=np.uint64)
    scale = d ** -0.5
    o, lse = attention.tree_attention(bf16.bf16_bits_to_f32(q), kval, vval, n_kv, tail, bits, scale,
                                      return_lse=True)
    out.update(parents=parents.astype(np.int32), bits=bits, tail=np.int64(tail), scale=np.float64(scale),
               out=o.astype(np.float32), lse=lse.astype(np.float32))
    return out


def main():
    for i, (m, n, k) in enumerate(QMM_CASES):
        np.savez_compressed(os.path.join(HERE, f"qmm_{i}.npz"), **qmm_fixture(i, m, n, k))
    for i, case in enumerate(ATTN_CASES):
        np.savez_compressed(os.path.join(HERE, f"attn_{i}.npz"), **attn_fixture(i, *case))
    anc_cases = {
        "reference_known_answer": np.array([-1, 0, 0], dtype=np.int32),  # tests/test_units.py:29-32
        "chain8": gen.chain_parents(8),
        "forest": np.array([-1, 0, -1, 2, 0, -1, 5, 1], dtype=np.int32),
        "random32": gen.tree_parents(np.random.default_rng(4000), 32),
        "random64": gen.tree_parents(np.random.default_rng(4001), 64),
    }
    np.savez_compressed(
        os.path.join(HERE, "ancestors.npz"),
        **{f"{k}_parents": v for k, v in anc_cases.items()},
        **{f"{k}_bits": tree.ancestor_bits_u64(v) for k, v in anc_cases.items()},
        **{f"{k}_depth": tree.depth(v) for k, v in anc_cases.items()},
    )
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
