"""Generate the golden fixtures in tests/golden/ from the UNMODIFIED reference.

The reference CPU kernels (src/ds3_reference.c of wzqhbustb/qw3) are built by
oracle/Makefile into oracle/_ref/libds3ref.so; this script feeds them small
seeded inputs and stores inputs + outputs as .npz files. The fixtures travel
with the repository, so the oracle restatement and the CUDA path can be
checked against the reference's own outputs on machines without the
reference sources.

Run from the repository root:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from qw3_b200 import inputs as I  # noqa: E402

OUT = Path(__file__).resolve().parent


def main() -> None:
    oracle.build()
    R = oracle.reference()
    if R is None:
        raise SystemExit("oracle/_ref/libds3ref.so not built (needs the reference sources)")

    # Embedding gather + dequant, both K-quant formats, two widths, with
    # repeated ids and the first/last rows of the table.
    for name, maker, type_ in (("q4k", I.q4k_table, 12), ("q6k", I.q6k_table, 14)):
        for n_cols, n_vocab, n_ids in ((512, 40, 24), (2048, 12, 6)):
            tab = maker(n_vocab, n_cols, 100 + n_cols)
            ids = I.token_ids(n_ids, 200 + n_cols, n_vocab)
            ids[0], ids[-1] = 0, n_vocab - 1
            if n_ids > 3:
                ids[2] = ids[1]
            rc, out = R.embed_rows(tab, type_, tab.shape[1], n_vocab, ids, n_cols)
            assert rc == 0
            w = I.gamma(n_cols, 300 + n_cols)
            rc, hid, nrm = R.embed_rms_norm(tab, type_, tab.shape[1], n_vocab, ids, n_cols, w, 1e-6)
            assert rc == 0 and np.array_equal(hid, out)
            np.savez_compressed(OUT / f"embed_{name}_{n_cols}.npz", table=tab, ids=ids, out=out, w=w,
                                norm=nrm, type=np.int32(type_), n_vocab=np.int32(n_vocab))

    # RMSNorm and residual add + RMSNorm.
    x = I.normal(400, (3, 2048))
    r = I.normal(401, (3, 2048))
    w = I.gamma(2048, 402)
    s, o = R.add_rms_norm(x, r, w, 1e-6)
    np.savez_compressed(OUT / "add_rms_norm.npz", x=x, r=r, w=w, sum=s, norm=o,
                        plain=R.rms_norm_rows(x, w, 1e-6))

    # Per-head QK norm + NEOX RoPE, including the largest long-context position.
    q = I.normal(500, (3, 32, 128))
    k = I.normal(501, (3, 4, 128))
    qw, kw = I.gamma(128, 502), I.gamma(128, 503)
    pos = np.array([0, 7, 32767], np.int32)
    qo, ko = R.qk_norm_rope(q, k, qw, kw, pos, 1e6, 1e-6)
    np.savez_compressed(OUT / "qk_norm_rope.npz", q=q, k=k, q_w=qw, k_w=kw, pos=pos, q_out=qo, k_out=ko,
                        q_rope_only=R.rope_rows(q, pos, 1e6))

    # Router softmax + top-8 + renorm.
    lg = I.normal(600, (16, 128), 0.0, 2.0)
    probs, idx, sc = R.router(lg, 8, True)
    _, idx_raw, sc_raw = R.router(lg, 8, False)
    np.savez_compressed(OUT / "router.npz", logits=lg, probs=probs, idx=idx, scores=sc, idx_raw=idx_raw,
                        scores_raw=sc_raw)

    # SwiGLU (weighted and plain) and the weighted combine + residual.
    g = I.normal(700, (8, 768), 0.0, 1.5)
    u = I.normal(701, (8, 768), 0.0, 1.5)
    rw = sc.reshape(-1)[:8].copy()
    np.savez_compressed(OUT / "swiglu.npz", gate=g, up=u, row_w=rw, out=R.swiglu(g, u, rw),
                        out_plain=R.swiglu(g, u, None))
    y = I.normal(800, (2 * 8, 1024))
    res = I.normal(801, (2, 1024))
    wts = sc[:2]
    np.savez_compressed(OUT / "combine.npz", y=y, w=wts, residual=res, out=R.combine(y, wts, res))

    # GGUF reader: the reference reader's header and tensor table for
    # synthetic model files (tests/gguf_writer.py, deterministic per config).
    import json
    import tempfile

    sys.path.insert(0, str(ROOT / "tests"))
    from gguf_writer import synthetic_model

    cases = []
    for cfg in (dict(), dict(alignment=256, embd_type=14, norm_type=0), dict(norm_type=8, n_layer=3, seed=3)):
        g, _ = synthetic_model(**cfg)
        with tempfile.TemporaryDirectory() as d:
            p = g.write(Path(d) / "m.gguf")
            ref = oracle.reference_gguf(p)
        assert ref and "error" not in ref
        for t in ref["tensors"]:
            t.pop("data_at")
        cases.append({"config": cfg, **ref})
    (OUT / "gguf_ref_table.json").write_text(json.dumps(cases, indent=1) + "\n")
    print("wrote fixtures to", OUT)


if __name__ == "__main__":
    main()
