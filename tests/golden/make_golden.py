"""Generate golden vectors by running the UNMODIFIED reference implementation.

Usage (only where the reference source tree is available; never on the GPU box):

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py \
        --reference <path-to-tao-memory-checkout> [case ...]

The reference is PyTorch + Triton.  On a machine without a GPU its Triton kernels
run under ``TRITON_INTERPRET=1``.  The Triton 3.6 interpreter has two defects
that this harness patches (the reference itself is not modified):

1. ``create_dot`` multiplies raw uint16 bit patterns of bf16 operands;
   the fix decodes bf16 to fp32 before ``np.matmul``.
2. fp32 -> bf16 casts truncate (and the rtne branch drops the carry), whereas
   the GPU backend rounds to nearest even; the fix routes the cast through
   torch's RTNE conversion.

With ``--fast`` the three inference kernels (query_fresh_fine, fusion scores,
fusion weighted sum) are replaced by torch restatements that were checked to be
bit-equal to the patched interpreter (see ``check_fast``); everything else, the
orchestration in particular, is the reference's own code.  Each fixture records
which mode produced it.

Outputs: ``tests/golden/<case>.pt`` (outputs only; inputs are regenerated from
the seed by ``oracle/inputs.py`` and guarded by a digest).
"""

import argparse
import os
import sys
import time

os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle.inputs import make_inputs, digest  # noqa: E402


def patch_interpreter():
    import triton.language as tl
    from triton.runtime import interpreter as interp

    builder = interp.InterpreterBuilder
    orig_dot = builder.create_dot

    def as_f32(x):
        return (x.astype(np.uint32) << 16).view(np.float32)

    def create_dot(self, a, b, d, input_precision, max_num_imprecise_acc):
        if a.dtype.scalar == tl.bfloat16 or b.dtype.scalar == tl.bfloat16:
            ad = as_f32(a.data) if a.dtype.scalar == tl.bfloat16 else a.data
            bd = as_f32(b.data) if b.dtype.scalar == tl.bfloat16 else b.data
            return interp.TensorHandle(np.matmul(ad, bd, dtype=d.data.dtype) + d.data,
                                       d.dtype.scalar)
        return orig_dot(self, a, b, d, input_precision, max_num_imprecise_acc)

    def to_bf16_bits(x):
        t = torch.from_numpy(np.ascontiguousarray(x).view(np.float32).copy())
        return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)

    orig_cast = builder.cast_impl
    orig_fp = builder.create_fp_to_fp

    def cast_impl(self, src, dst_type):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return interp.TensorHandle(to_bf16_bits(src.data), dst_type.scalar)
        return orig_cast(self, src, dst_type)

    def create_fp_to_fp(self, src, dst_type, rounding_mode):
        if src.dtype.scalar == tl.float32 and dst_type.scalar == tl.bfloat16:
            return interp.TensorHandle(to_bf16_bits(src.data), dst_type.scalar)
        return orig_fp(self, src, dst_type, rounding_mode)

    builder.create_dot = create_dot
    builder.cast_impl = cast_impl
    builder.create_fp_trunc = lambda self, src, dst_type: self.cast_impl(src, dst_type)
    builder.create_fp_to_fp = create_fp_to_fp


def install_fast(ref):
    """Swap the three inference Triton kernels for bit-equal torch restatements."""
    sys.path.insert(0, os.path.dirname(HERE))
    from oracle import tao_oracle as o
    import tao_attention.query_fresh_fine as qff
    import tao_attention.operator as op

    qff.query_fresh_fine_parts = o.fine_read
    qff.query_fresh_fine_read = lambda *a, **k: o.fine_read(*a, **k)[-1]
    op.fusion_scores = o.fusion_scores
    op.fusion_weighted_sum = o.fusion_weighted_sum


def check_fast():
    """The restatements agree bit-for-bit with the patched interpreter."""
    import tao_attention.query_fresh_fine as qff
    import tao_attention.fusion_pointwise as fp
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from oracle import tao_oracle as o
    g = torch.Generator().manual_seed(7)
    b, q, h, p, d, s, m = 1, 3, 2, 4, 64, 30, 7
    hv = torch.rand(b, q, h, p, d, generator=g).to(torch.bfloat16) * 0.05
    pz = torch.randn(b, h, p, d, generator=g).to(torch.bfloat16) + 5
    fz = torch.randn(b, h, s, d, generator=g).to(torch.bfloat16) + 4
    ids = torch.randint(0, s, (b, 1, h, m), generator=g)
    fc = torch.randn(b, h, s, d, d, generator=g).to(torch.bfloat16)
    ref = qff.query_fresh_fine_parts(hv, pz, fz, ids.expand(b, q, h, m), fc, 8)
    mine = o.fine_read(hv, pz, fz, ids, fc, 8)
    for x, y in zip(ref, mine):
        assert torch.equal(x, y), "fine read restatement differs"
    rq = torch.randn(1, 5, h, d, generator=g).to(torch.bfloat16)
    fa = (torch.randn(h, d, 3, generator=g) * 0.02)
    fb = (torch.randn(h, d, 3, generator=g) * 0.02)
    for c, f in ((False, True), (False, False), (True, True)):
        assert torch.equal(fp.fusion_scores(rq, fa, fb, c, f), o.fusion_scores(rq, fa, fb, c, f))
    rho = torch.softmax(o.fusion_scores(rq, fa, fb, False, True).float(), -1).to(torch.bfloat16)
    loc, fin = (torch.randn(1, 5, h, d, generator=g).to(torch.bfloat16) for _ in range(2))
    gain = torch.full((), 0.8, dtype=torch.bfloat16)
    assert torch.equal(fp.fusion_weighted_sum(rho, loc, torch.zeros_like(fin), fin, gain),
                       o.fusion_weighted_sum(rho, loc, torch.zeros_like(fin), fin, gain))
    print("fast restatements: bit-equal to the patched interpreter")


# ---------------------------------------------------------------------------

STREAM_CASES = {
    # name: (heads, width, layer_index, prefill split, decode steps, seed)
    "stream_h2d64": (2, 64, 1, (700, 1000, 1116), 48, 1),
    "stream_h1d128": (1, 128, 0, (1300,), 30, 2),
    "stream_pages": (1, 64, 3, (9000,), 40, 3),
}

# streaming cases with another fine writer on the index-only preset:
# name: (case tuple as above, fine_writer)
WRITER_CASES = {
    "stream_regularized": ((2, 64, 1, (1000, 1900), 40, 8), "regularized_association"),
    "stream_feature_mass": ((2, 64, 1, (1000, 1900), 40, 11), "feature_mass_association"),
    "stream_structured_gram": ((2, 64, 1, (1000, 1900), 40, 13), "structured_gram_association"),
}

# training cases with another fine writer on the index-only preset
TRAIN_WRITER_CASES = {
    "train_regularized": ((1, 2048, 2, 64, 0.5, 9), "regularized_association"),
    "train_feature_mass": ((1, 2048, 2, 64, 0.5, 23), "feature_mass_association"),
    "train_structured_gram": ((1, 3072, 1, 64, 0.4, 24), "structured_gram_association"),
}

# cases on the historical default TaoConfig() (coarse_index_only=False: completed
# pages carry a coarse value matrix that every query reads), softmax writer
DEFAULT_CONFIG_STREAM_CASES = {
    "stream_coarse": (2, 64, 1, (1500, 1800, 1600), 40, 14),
}
DEFAULT_CONFIG_TRAIN_CASES = {
    "train_coarse": (1, 4608, 1, 64, 0.6, 15),
}

TRAIN_CASES = {
    # name: (batch, tokens, heads, width, alpha, seed)
    "train_t2048_h2": (1, 2048, 2, 64, 0.5, 4),
    "train_t3072_b2": (2, 3072, 1, 64, 0.3, 5),
    "train_t2000_ragged": (1, 2000, 1, 64, 0.7, 6),
    "train_pages": (1, 9216, 1, 64, 0.5, 7),
}


def run_stream(name, mode):
    from tao_attention import new_state, tao_attention_prefill, tao_attention_decode, StreamCache
    from tao_attention.presets import index_only_page_memo
    from tao_attention.config import TaoConfig
    if name in WRITER_CASES:
        case, writer = WRITER_CASES[name]
        base = index_only_page_memo()
        config = TaoConfig(**{**base.export(), "fine_writer": writer})
    elif name in DEFAULT_CONFIG_STREAM_CASES:
        case, config = DEFAULT_CONFIG_STREAM_CASES[name], TaoConfig()
    else:
        case, config = STREAM_CASES[name], index_only_page_memo()
    heads, width, layer, splits, steps, seed = case
    total = sum(splits) + steps
    x, _ = make_inputs(1, total, heads, width, seed)
    alpha = 0.5
    state = new_state(layer, config)
    outs, route_ids, positions = [], [], []
    pos = 0
    kw = dict(fusion_a=x["fusion_a"], fusion_b=x["fusion_b"], alpha=alpha)
    with torch.inference_mode():
        for n in splits:
            sl = slice(pos, pos + n)
            out, state = tao_attention_prefill(x["q"][:, sl], x["k"][:, sl], x["v"][:, sl],
                                               raw_q=x["raw_q"][:, sl], raw_k=x["raw_k"][:, sl],
                                               state=state, position=pos, **kw)
            outs.append(out)
            pos += n
        prefill_ids = state.layers[0].route_ids
        snap_at = steps // 2
        snapshot = None
        for i in range(steps):
            sl = slice(pos, pos + 1)
            out, state = tao_attention_decode(x["q"][:, sl], x["k"][:, sl], x["v"][:, sl],
                                              raw_q=x["raw_q"][:, sl], raw_k=x["raw_k"][:, sl],
                                              state=state, position=pos, **kw)
            outs.append(out)
            ids = state.layers[0].route_ids
            route_ids.append(None if ids is None else ids[1].clone())
            positions.append(pos)
            pos += 1
            if i + 1 == snap_at:
                snapshot = state.export()
        final = state.export()
    return {
        "kind": "stream", "mode": mode, "case": case, "alpha": alpha, "config": config.export(),
        "input_digest": digest(*(x[k] for k in ("q", "k", "v", "raw_q", "raw_k", "fusion_a", "fusion_b"))),
        "output": torch.cat(outs, dim=1),
        "prefill_route_ids": None if prefill_ids is None else prefill_ids[1].clone(),
        "decode_route_ids": route_ids, "decode_positions": positions,
        "snapshot_mid": snapshot, "snapshot_final": final,
        "bytes": state.bytes(),
    }


def run_train(name, mode):
    from tao_attention import tao_attention
    from tao_attention.presets import index_only_page_memo
    from tao_attention.config import TaoConfig
    if name in TRAIN_WRITER_CASES:
        case, writer = TRAIN_WRITER_CASES[name]
        config = TaoConfig(**{**index_only_page_memo().export(), "fine_writer": writer})
    elif name in DEFAULT_CONFIG_TRAIN_CASES:
        case, config = DEFAULT_CONFIG_TRAIN_CASES[name], TaoConfig()
    else:
        case, config = TRAIN_CASES[name], index_only_page_memo()
    batch, tokens, heads, width, alpha, seed = case
    x, g = make_inputs(batch, tokens, heads, width, seed)
    grad = torch.randn(batch, tokens, heads, width, generator=g).to(torch.bfloat16)
    leaves = {k: x[k].clone().requires_grad_(True) for k in x}
    out = tao_attention(leaves["q"], leaves["k"], leaves["v"], raw_q=leaves["raw_q"],
                        raw_k=leaves["raw_k"], fusion_a=leaves["fusion_a"],
                        fusion_b=leaves["fusion_b"], alpha=alpha,
                        config=config)
    out.backward(grad)
    return {
        "kind": "train", "mode": mode, "case": case, "alpha": alpha, "config": config.export(),
        "input_digest": digest(*(x[k] for k in ("q", "k", "v", "raw_q", "raw_k", "fusion_a", "fusion_b")), grad),
        "output": out.detach(),
        "grads": {k: leaves[k].grad.detach().clone() for k in leaves},
    }


# Row subsampling applied before saving, to keep the committed fixtures small.
STRIDE = {"train_pages": 4, "train_t3072_b2": 2, "train_t2048_h2": 2, "stream_pages": 3,
          "stream_h2d64": 2, "stream_coarse": 2, "train_coarse": 2}


def compact(name, result):
    stride = STRIDE.get(name, 1)
    result["row_stride"] = stride
    if stride == 1:
        return result
    if result["kind"] == "train":
        result["output"] = result["output"][:, ::stride].clone()
        for k in ("q", "k", "v", "raw_q", "raw_k"):
            result["grads"][k] = result["grads"][k][:, ::stride].clone()
    else:
        steps = (WRITER_CASES[name][0] if name in WRITER_CASES else
                 DEFAULT_CONFIG_STREAM_CASES.get(name) or STREAM_CASES[name])[4]
        out = result["output"]
        result["decode_output"] = out[:, -steps:].clone()
        result["output"] = out[:, ::stride].clone()
        result["snapshot_mid"] = None
    return result


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ap.add_argument("--fast", action="store_true")
    ap.add_argument("--threads", type=int, default=1)
    ap.add_argument("--compact-only", action="store_true",
                    help="re-apply the row subsampling to existing full fixtures")
    ap.add_argument("cases", nargs="*")
    args = ap.parse_args()
    torch.set_num_threads(args.threads)
    sys.path.insert(0, os.path.abspath(args.reference))
    patch_interpreter()
    if args.fast:
        check_fast()
        install_fast(args.reference)
    mode = "reference+fast-inference-kernels" if args.fast else "reference (interpreted Triton, patched)"
    cases = args.cases or [*STREAM_CASES, *WRITER_CASES, *TRAIN_CASES, *TRAIN_WRITER_CASES,
                           *DEFAULT_CONFIG_STREAM_CASES, *DEFAULT_CONFIG_TRAIN_CASES]
    if args.compact_only:
        for name in cases:
            path = os.path.join(HERE, name + ".pt")
            result = torch.load(path, weights_only=False)
            if "row_stride" not in result:
                torch.save(compact(name, result), path)
        return
    for name in cases:
        t0 = time.time()
        streaming = name in STREAM_CASES or name in WRITER_CASES or name in DEFAULT_CONFIG_STREAM_CASES
        result = run_stream(name, mode) if streaming else run_train(name, mode)
        torch.save(compact(name, result), os.path.join(HERE, name + ".pt"))
        print(f"{name}: {time.time() - t0:.1f}s ({mode})", flush=True)


if __name__ == "__main__":
    main()
