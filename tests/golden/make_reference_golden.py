"""Generates tests/golden/reference_golden.npz by EXECUTING the reference's own source.

The unmodified files of aabhimittal/TPU-Native-Pallas-FlashAttention
(``src/pallas_flash/{reference,flash_attention,fused_rope,paged,model,config}.py``
and the helpers of ``tests/test_paged.py``) are loaded from the reference
checkout and run under ``jax_numpy_shim`` (numpy stand-ins for the jax names
they use; ``pallas_call`` executes each Pallas kernel body grid point by grid
point, as interpret mode does).  The reference's float32 arithmetic is carried
out in float64 (``jax_numpy_shim.WIDE``), so the stored outputs are the
reference algorithm's results to float64 accuracy, then rounded to float32.

Inputs are NOT stored: ``golden_inputs.py`` rebuilds them from (shape, seed)
with a library-independent counter-based generator (bfloat16-representable
N(0, 1) values as float32, so one fixture serves the fp32 and the bf16 kernel
tests); the file holds the reference's outputs, the block tables the
reference's test helper drew, and the gathered caches as bfloat16 bits.
Every output comes from the reference's own code path:

* ``fwd/*``     ``_flash_attention_call`` (out and LSE), the Pallas forward kernel
                (flash_attention.py:61-227), and ``reference_attention``
                (reference.py:22-66) on the same inputs;
* ``bwd/*``     ``_flash_attention_vjp_fwd`` + ``_flash_attention_vjp_bwd``: the
                delta preprocess, dQ and dK/dV Pallas kernels with the GQA
                group-sum (flash_attention.py:245-476);
* ``dec/*``     ``flash_attention_decode`` (flash_attention.py:555-589);
* ``rope/*``    ``flash_attention_rope`` (fused_rope.py:53-213) with tables from
                ``model.precompute_rope`` (model.py:41-52);
* ``paged/*``   ``paged_flash_attention`` (paged.py:45-192) over
                ``tests/test_paged.py:_scrambled_table`` tables, the
                ``_gather_contiguous`` helper (test_paged.py:25-28) and
                ``write_to_paged_cache`` (paged.py:205-223);
* ``model/*``   ``rms_norm``, ``apply_rope``, ``swiglu_mlp``, ``forward``,
                ``generate``, ``generate_cached`` and ``generate_streaming``
                (model.py:34-531) with ``init_params`` run through the shim's
                numpy ``jax.random``; the parameters are stored.

Run here, where the reference checkout exists (it does not exist on the GPU
hosts; the tests read only the .npz):

    python tests/golden/make_reference_golden.py [--reference PATH]
"""

from __future__ import annotations

import argparse
import importlib
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
OUT = HERE / "reference_golden.npz"
DEFAULT_REF = Path("/root/reference")


def load_reference(ref_root: Path):
    """Imports the reference package (and its paged test module) under the shim."""
    sys.path.insert(0, str(HERE))
    import jax_numpy_shim
    jax_numpy_shim.install(wide=True)
    for name in list(sys.modules):
        if name == "pallas_flash" or name.startswith("pallas_flash."):
            del sys.modules[name]
    pkg_dir = ref_root / "src" / "pallas_flash"
    spec = importlib.util.spec_from_file_location("pallas_flash", pkg_dir / "__init__.py",
                                                  submodule_search_locations=[str(pkg_dir)])
    pkg = importlib.util.module_from_spec(spec)
    sys.modules["pallas_flash"] = pkg
    spec.loader.exec_module(pkg)
    tspec = importlib.util.spec_from_file_location("ref_test_paged", ref_root / "tests" / "test_paged.py")
    tmod = importlib.util.module_from_spec(tspec)
    tspec.loader.exec_module(tmod)
    return pkg, tmod, jax_numpy_shim


def f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float64).astype(np.float32)


def bf16_bits(x) -> np.ndarray:
    """float32 values that are bfloat16-representable -> their uint16 bit patterns."""
    return (np.ascontiguousarray(x, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=DEFAULT_REF)
    args = ap.parse_args()
    pf, tpaged, shim = load_reference(args.reference)
    import golden_inputs as gi
    fa = sys.modules["pallas_flash.flash_attention"]
    mdl = sys.modules["pallas_flash.model"]
    out: dict[str, np.ndarray] = {}
    W = lambda x: np.asarray(x, np.float64).view(shim.Arr)  # noqa: E731  inputs to the reference

    # ---------------- forward kernel + naive reference ---------------------- #
    for case in gi.FWD_CASES:
        name, B, H, Hkv, Sq, Sk, D, causal, kv_len, bq, bk, seed = case
        q, k, v = gi.fwd_inputs(case)
        o, lse = fa._flash_attention_call(
            W(q), W(k), W(v), causal=causal, sm_scale=1.0 / D ** 0.5, block_q=bq, block_k=bk,
            kv_len=Sk if kv_len is None else kv_len, interpret=True)
        p = f"fwd/{name}/"
        out.update({p + "o": f32(o), p + "lse": f32(lse)})
        if kv_len is None and q.size <= 1 << 16:
            out[p + "naive"] = f32(pf.reference_attention(W(q), W(k), W(v), causal=causal))

    # ---------------- backward kernels (custom_vjp rules) ------------------- #
    for case in gi.BWD_CASES:
        name, B, H, Hkv, S, D, causal, bq, bk, seed = case
        q, k, v, do = gi.bwd_inputs(case)
        o, res = fa._flash_attention_vjp_fwd(causal, 1.0 / D ** 0.5, bq, bk, S, True, W(q), W(k), W(v))
        dq, dk, dv = fa._flash_attention_vjp_bwd(causal, 1.0 / D ** 0.5, bq, bk, S, True, res, W(do))
        p = f"bwd/{name}/"
        out.update({p + "dq": f32(dq), p + "dk": f32(dk), p + "dv": f32(dv)})

    # ---------------- fixed-cache decode ------------------------------------ #
    for n_kv in gi.DEC_KV:
        q, kc, vc = gi.dec_inputs(n_kv)
        for cache_len in gi.DEC_LENS:
            o = pf.flash_attention_decode(W(q), W(kc), W(vc), cache_len, interpret=True)
            out[f"dec/kv{n_kv}_len{cache_len}/o"] = f32(o)
    # the NaN-tail known answer of test_decode.py:38-49, run through the reference
    filled = 8
    kn = np.concatenate([np.ones((1, 2, filled, 128)), np.full((1, 2, 120, 128), np.nan)], axis=2)
    o = pf.flash_attention_decode(W(np.ones((1, 2, 1, 128))), W(kn), W(kn), filled, interpret=True)
    out["dec/nan_tail/o"] = f32(o)

    # ---------------- fused RoPE -------------------------------------------- #
    theta = 10000.0
    for case in gi.ROPE_CASES:
        name, B, H, Hkv, S, causal, seed = case
        q, k, v = gi.rope_inputs(case)
        cos, sin = mdl.precompute_rope(S, 128, theta)
        o = pf.flash_attention_rope(W(q), W(k), W(v), cos, sin, causal=causal, interpret=True)
        out[f"rope/{name}/o"] = f32(o)
    pos, cache = 77, 128  # one query at absolute position 77, keys [0, 77] (test_fused_rope.py:53-70)
    q, k, v = gi.rope_decode_inputs()
    cos, sin = mdl.precompute_rope(cache, 128, theta)
    o = pf.flash_attention_rope(W(q), W(k), W(v), cos[pos:pos + 1], sin[pos:pos + 1], cos, sin,
                                causal=False, block_q=1, kv_len=pos + 1, interpret=True)
    out["rope/decode_pos77/o"] = f32(o)
    for S, D in ((300, 128), (64, 64)):
        cos, sin = mdl.precompute_rope(S, D, theta)
        out[f"rope/table_s{S}_d{D}/cos"], out[f"rope/table_s{S}_d{D}/sin"] = f32(cos), f32(sin)

    # ---------------- paged decode + page helpers ---------------------------- #
    for i, (B, H, Hkv, ps, lens) in enumerate(gi.PAGED_CASES):
        num_pages, D = 32, 128
        pps = max(lens) // ps + 1
        q, kp, vp = gi.paged_inputs(i)
        table = np.asarray(tpaged._scrambled_table(B, pps, num_pages, seed=B), np.int32)
        ln = np.asarray(lens, np.int32)
        o = pf.paged_flash_attention(W(q), W(kp), W(vp), table, ln, interpret=True)
        gathered = np.zeros((B, Hkv, max(lens), D), np.float32)
        for b, length in enumerate(lens):
            gathered[b, :, :length] = f32(tpaged._gather_contiguous(W(kp), table[b], pps, length))
        p = f"paged/case{i}/"
        out.update({p + "table": table, p + "o": f32(o), p + "k_gathered_bf16": bf16_bits(gathered)})
    ps, D, n_kv, num_pages, length = 32, 128, 2, 4, 70  # test_paged.py:94-113
    kpool, vpool = pf.init_paged_cache(num_pages, n_kv, ps, D)
    table = np.asarray([0, 2, 1, 3], np.int32)
    kseq, vseq, q = gi.paged_write_inputs()
    for t in range(length):
        kpool, vpool = pf.write_to_paged_cache(kpool, vpool, W(kseq[:, :, t:t + 1]),
                                               W(vseq[:, :, t:t + 1]), table, t)
    o = pf.paged_flash_attention(W(q), kpool, vpool, table[None], np.asarray([length], np.int32),
                                 interpret=True)
    out.update({"paged/write/table": table, "paged/write/k_pool_bf16": bf16_bits(f32(kpool)),
                "paged/write/v_pool_bf16": bf16_bits(f32(vpool)), "paged/write/o": f32(o)})

    # ---------------- model building blocks and generation ------------------- #
    x, w = gi.randn((2, 5, 64), 700), gi.randn((64,), 701)
    out["model/rms/y"] = f32(mdl.rms_norm(W(x), W(w), 1e-5))
    cos, sin = mdl.precompute_rope(64, 64, theta)
    out["model/rope/y"] = f32(mdl.apply_rope(W(gi.randn((2, 3, 64, 64), 702)), cos, sin))
    xs = gi.randn((3, 64), 703)
    wg, wu, wd = (gi.randn((64, 96), 704) * 0.125, gi.randn((64, 96), 705) * 0.125,
                  gi.randn((96, 64), 706) * 0.125)
    out["model/mlp/y"] = f32(mdl.swiglu_mlp(W(xs), W(wg), W(wu), W(wd)))

    for case in gi.MODEL_CASES:
        name, H, Hkv, hd, ffn, nl, prompt, n_new, window, seed = case
        cfg = pf.ModelConfig(vocab_size=64, dim=H * hd, n_layers=nl, n_heads=H, n_kv_heads=Hkv,
                             head_dim=hd, ffn_hidden=ffn, max_seq_len=256)
        params = gi.model_params(case)
        wp = {k2: ([{a: W(b) for a, b in lay.items()} for lay in v2] if k2 == "layers" else W(v2))
              for k2, v2 in params.items()}
        pr = np.asarray(prompt, np.int64)
        p = f"model/{name}/"
        out[p + "logits"] = f32(mdl.forward(wp, pr, cfg, interpret=True))
        toks_full = mdl.generate(wp, pr, n_new, cfg, interpret=True)
        toks_cached = mdl.generate_cached(wp, pr, n_new, cfg, interpret=True)
        toks_stream = mdl.generate_streaming(wp, pr, n_new, cfg, window=window, interpret=True)
        assert np.array_equal(toks_full, toks_cached), name
        out[p + "tokens_cached"] = np.asarray(toks_cached, np.int64)
        out[p + "tokens_stream"] = np.asarray(toks_stream, np.int64)
        margins, seq = [], pr  # top-1 minus top-2 logit at every greedy step of the cached path
        for _ in range(n_new):
            lg = np.asarray(mdl.forward(wp, seq, cfg, interpret=True))[:, -1, :]
            srt = np.sort(lg, axis=-1)
            margins.append(srt[:, -1] - srt[:, -2])
            seq = np.concatenate([seq, np.argmax(lg, axis=-1)[:, None]], axis=1)
        out[p + "margin_min"] = np.array([np.min(margins)], np.float64)
        print(f"{name}: cached {np.asarray(toks_cached)[:, pr.shape[1]:].tolist()} "
              f"stream {np.asarray(toks_stream)[:, pr.shape[1]:].tolist()} min margin {np.min(margins):.4f}")
    out["model/ring_kv_len"] = np.array([mdl.ring_kv_len(t, c) for t, c in
                                         ((3, 8), (8, 8), (50, 8), (1, 8))], np.int64)

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size / 1e6:.2f} MB, {len(out)} arrays)")


if __name__ == "__main__":
    main()
