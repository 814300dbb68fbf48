"""Generate golden vectors by running the reference implementation itself.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/msa_triton

The reference is imported in place through a temporary ``msa_triton`` symlink;
only its pure-torch parts run here (eager ops, the FP64 oracle
tests/reference_fp64.py, triton/topk.py and triton/k2q.py, which do not need
Triton). Outputs are small ``.npz`` files next to this script; tests load them
on any machine without the reference. Inputs are stored as float32 arrays
holding exactly the bf16/fp16/fp32 values that were fed to the reference.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))


def import_reference(path: str):
    tmp = tempfile.mkdtemp(prefix="msa_ref_")
    os.symlink(path, os.path.join(tmp, "msa_triton"))
    sys.path.insert(0, tmp)
    os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
    sys.dont_write_bytecode = True
    import msa_triton.eager as eager  # noqa: F401
    from msa_triton.tests import reference_fp64
    from msa_triton.triton import topk as ref_topk
    from msa_triton.triton import k2q as ref_k2q
    return eager, reference_fp64, ref_topk, ref_k2q


def cu_of(lengths):
    return torch.tensor([0, *torch.tensor(lengths, dtype=torch.int64).cumsum(0).tolist()], dtype=torch.int32)


def f32(x):
    return x.detach().to(torch.float32).numpy()


def f64(x):
    return x.detach().to(torch.float64).numpy()


DTYPE_NAME = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}


# ---------------------------------------------------------------- index score
def score_cases():
    """(name, lengths, G, Di, B, scale, seed, dtype, max_seqlen_extra)."""
    cases = []
    for i, (lengths, g, d, b, s) in enumerate([
        ([1], 1, 1, 4, 1.0), ([0, 0], 2, 7, 4, 1.0), ([0, 3, 0, 2, 0], 2, 7, 4, 1.0),
        ([3, 7], 2, 7, 4, 1.0), ([7, 11], 4, 16, 8, 0.5), ([9], 2, 64, 4, 1.0),
        ([5], 4, 128, 128, 1.0), ([127, 129], 3, 16, 128, 1.0), ([257], 2, 64, 128, 0.125),
        ([40, 3], 2, 64, 16, -0.75),
    ]):
        cases.append((f"rand{i}", lengths, g, d, b, s, 731 + i, torch.bfloat16))
    cases.append(("f16", [2, 0, 4], 2, 7, 4, 0.3, 928, torch.float16))
    cases.append(("f32", [2, 0, 4], 2, 7, 4, 0.3, 929, torch.float32))
    return cases


def gen_score(ref_fp64, eager):
    out = {}
    meta = []
    for name, lengths, g, d, b, scale, seed, dtype in score_cases():
        gen = torch.Generator().manual_seed(seed)
        t = sum(lengths)
        q = torch.randn(t, g, d, generator=gen).to(dtype)
        k = torch.randn(t, 1, d, generator=gen).to(dtype)
        max_seqlen = max(max(lengths), 1) + b
        cu = cu_of(lengths)
        qr, kr = q.double().requires_grad_(), k.double().requires_grad_()
        s = ref_fp64.index_score_fp64(qr, kr, cu, max_seqlen, block_size=b, scale=scale)
        up = torch.randn(s.shape, generator=gen).to(torch.bfloat16).double()
        s.backward(up)
        es = eager.m3_index_score(q, k, cu, max_seqlen, block_size=b, scale=scale)
        out[f"{name}/iq"], out[f"{name}/ik"] = f32(q), f32(k)
        out[f"{name}/cu"] = cu.numpy()
        out[f"{name}/scores"] = f64(s)
        out[f"{name}/eager_scores"] = f32(es)
        out[f"{name}/dscores"] = f64(up)
        out[f"{name}/diq"], out[f"{name}/dik"] = f64(qr.grad), f64(kr.grad)
        meta.append(dict(name=name, lengths=lengths, groups=g, dim=d, block_size=b, scale=scale,
                         max_seqlen=max_seqlen, dtype=DTYPE_NAME[dtype]))
    # Known answers: exact ties split equally (reference test_triton_score.py:93-108,
    # test_eager.py:56-65) and low-bit winners (test_triton_score.py:133-182).
    kat = []
    for scale in (1.0, 0.0, -1.0):
        kat.append((f"tie_s{scale:+.0f}", torch.ones(5, 2, 3), torch.ones(5, 1, 3), [2, 3], 4, 8, scale,
                    torch.bfloat16, "ones"))
    small = 2 ** -12
    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        for scale in (1.0, -1.0, 0.0):
            for case in ("cancellation_unique", "cancellation_tie", "rounded_score_tie"):
                if case.startswith("cancellation"):
                    query = [1.0, small, 1.0]
                    key0 = [1.0, small, -1.0]
                    key1 = [0.0, small if case.endswith("tie") else 0.0, 0.0]
                else:
                    query, key0, key1 = [1.0, 1.0], [1.0, 2 ** -24], [1.0, 0.0]
                kat.append((f"{case}_{DTYPE_NAME[dtype]}_s{scale:+.0f}", torch.tensor([[query], [query]]),
                            torch.tensor([[key0], [key1]]), [2], 2, 2, scale, dtype, "row1"))
    for exact_tie in (False, True):
        query = [1 + 2 ** -12, 1.0]
        k0 = [[1 + 2 ** -12, -1 - 2 ** -11]]
        k1 = [[0.0, 2 ** -24 if exact_tie else 0.0]]
        kat.append((f"residual_tie{int(exact_tie)}", torch.tensor([[query], [query]]),
                    torch.tensor([k0, k1]), [2], 2, 2, 1.0, torch.float32, "row1"))
    for name, q, k, lengths, b, max_seqlen, scale, dtype, upstream in kat:
        q, k = q.to(dtype), k.to(dtype)
        cu = cu_of(lengths)
        qr, kr = q.double().requires_grad_(), k.double().requires_grad_()
        s = ref_fp64.index_score_fp64(qr, kr, cu, max_seqlen, block_size=b, scale=scale)
        if upstream == "ones":
            up = torch.ones_like(s)
        else:
            up = torch.zeros_like(s)
            up[1] = 1
        s.backward(up)
        out[f"{name}/iq"], out[f"{name}/ik"] = f32(q), f32(k)
        out[f"{name}/cu"] = cu.numpy()
        out[f"{name}/scores"] = f64(s)
        out[f"{name}/eager_scores"] = f32(eager.m3_index_score(q, k, cu, max_seqlen, block_size=b, scale=scale))
        out[f"{name}/dscores"] = f64(up)
        out[f"{name}/diq"], out[f"{name}/dik"] = f64(qr.grad), f64(kr.grad)
        meta.append(dict(name=name, lengths=lengths, groups=q.shape[1], dim=q.shape[2], block_size=b,
                         scale=scale, max_seqlen=max_seqlen, dtype=DTYPE_NAME[dtype]))
    return out, meta


# ---------------------------------------------------------------- top-k
def gen_topk(eager, ref_topk):
    out, meta = {}, []
    params = [([1, 7, 3], 2, 3, 1), ([127, 128, 129], 128, 16, 1), ([17, 0, 9], 4, 2, 0),
              ([8, 5], 2, 3, 3), ([2], 1, 0, 0), ([300, 45], 16, 5, 2), ([400], 8, 32, 2)]
    for i, (lengths, block, k, local) in enumerate(params):
        cu = cu_of(lengths)
        groups, blocks = 3, (max(lengths) + block - 1) // block
        scores = torch.randn(sum(lengths), groups, blocks, generator=torch.Generator().manual_seed(82 + i))
        if i == 5:  # exact ties among ranked candidates
            scores = scores.round()
        name = f"case{i}"
        out[f"{name}/scores"] = scores.numpy()
        out[f"{name}/cu"] = cu.numpy()
        out[f"{name}/eager"] = eager.m3_topk(scores, cu, block_size=block, topk_blocks=k, local_blocks=local).numpy()
        out[f"{name}/native"] = ref_topk.m3_topk(scores, cu, block_size=block, topk_blocks=k, local_blocks=local).numpy()
        meta.append(dict(name=name, lengths=lengths, block_size=block, topk_blocks=k, local_blocks=local))
    # all-equal scores with local forcing (reference test_topk.py:53-66)
    scores = torch.zeros(7, 2, 4)
    cu = cu_of([7])
    out["equal/scores"], out["equal/cu"] = scores.numpy(), cu.numpy()
    out["equal/eager"] = eager.m3_topk(scores, cu, block_size=2, topk_blocks=2, local_blocks=1).numpy()
    out["equal/native"] = ref_topk.m3_topk(scores, cu, block_size=2, topk_blocks=2, local_blocks=1).numpy()
    meta.append(dict(name="equal", lengths=[7], block_size=2, topk_blocks=2, local_blocks=1))
    return out, meta


# ---------------------------------------------------------------- k2q
def gen_k2q(ref_k2q):
    out, meta = {}, []
    params = [([1], 1, 4, 128), ([3, 5], 3, 5, 2), ([0, 3, 0, 2, 0], 2, 4, 2),
              ([127, 128, 129], 4, 5, 128), ([0, 0], 3, 5, 128), ([4, 2], 3, 0, 2),
              ([600, 77, 300], 4, 6, 16)]
    cases = []
    for i, (lengths, groups, slots, b) in enumerate(params):
        max_blocks = (max(lengths) + b - 1) // b
        ids = torch.randint(-2, max_blocks + 4, (sum(lengths), groups, slots),
                            generator=torch.Generator().manual_seed(951 + i), dtype=torch.int32)
        cases.append((f"rand{i}", ids, lengths, b))
    ids = torch.tensor([[[0, 0, 1], [1, 0, -1]], [[0, -1, 8], [0, 0, 1]], [[1, 0, 1], [0, 1, -2]],
                        [[0, 0, 1], [0, -1, 9]], [[0, 0, -1], [0, 0, -1]]], dtype=torch.int32)
    cases.append(("duplicates", ids, [3, 2], 2))
    lengths, groups, slots, b = [9, 5], 4, 3, 4
    ids = torch.full((sum(lengths), groups, slots), -1, dtype=torch.int32)
    start = 0
    for length in lengths:
        for local in range(length):
            ids[start + local, :, 0] = local // b
            ids[start + local, :, 1] = 0
            if local // b > 0:
                ids[start + local, :, 2] = local // b - 1
        start += length
    cases.append(("hotspots", ids, lengths, b))
    ids = torch.full((7, 2, 4), 99, dtype=torch.int32)
    ids[:, :, 0] = -1
    cases.append(("all_invalid", ids, [3, 4], 2))
    for name, ids, lengths, b in cases:
        cu = cu_of(lengths)
        r = ref_k2q.build_k2q_csr(ids, cu, block_size=b)
        out[f"{name}/indices"], out[f"{name}/cu"] = ids.numpy(), cu.numpy()
        out[f"{name}/row_ptr"] = r.row_ptr.numpy()
        out[f"{name}/query_indices"] = r.query_indices.numpy()
        out[f"{name}/slot_indices"] = r.slot_indices.numpy()
        out[f"{name}/cu_block_lens"] = r.cu_block_lens.numpy()
        meta.append(dict(name=name, lengths=lengths, block_size=b))
    return out, meta


# ---------------------------------------------------------------- attention
def attention_indices(lengths, groups, block_size, topk):
    """The selection pattern of the reference's attention tests (test_triton_attention.py:42-54)."""
    total = sum(lengths)
    indices = torch.full((total, groups, topk), -1, dtype=torch.int32)
    start = 0
    for length in lengths:
        for offset in range(length):
            for group in range(groups):
                current = offset // block_size
                cand = [current] + [b for b in range(current) if (b + group) % 2 == 0]
                chosen = cand[:topk]
                if chosen:
                    indices[start + offset, group, :len(chosen)] = torch.tensor(chosen, dtype=torch.int32)
        start += length
    return indices


def gen_attention(ref_fp64, eager):
    out, meta = {}, []
    params = [
        ([1], 1, 1, 5, 128, 1, None), ([7, 3], 2, 2, 8, 3, 3, None), ([17, 5], 3, 1, 16, 8, 2, 0.2),
        ([129, 1], 1, 2, 8, 128, 3, None), ([127, 128, 257], 1, 1, 8, 128, 3, None),
        ([5, 1, 9], 2, 4, 32, 4, 4, None), ([5, 3], 2, 2, 128, 4, 2, None),
        ([0, 3, 0, 2, 0], 2, 2, 8, 2, 2, None), ([140], 1, 2, 128, 128, 2, None),
        ([130, 20], 2, 2, 64, 64, 3, -0.3),
    ]
    for i, (lengths, groups, ratio, dim, b, topk, scale) in enumerate(params):
        gen = torch.Generator().manual_seed(1234 + i)
        total = sum(lengths)
        q = torch.randn(total, groups * ratio, dim, generator=gen).to(torch.bfloat16)
        k = torch.randn(total, groups, dim, generator=gen).to(torch.bfloat16)
        v = torch.randn(total, groups, dim, generator=gen).to(torch.bfloat16)
        go = torch.randn(total, groups * ratio, dim, generator=gen).to(torch.bfloat16)
        ids = attention_indices(lengths, groups, b, topk)
        cu = cu_of(lengths)
        refs = [x.double().requires_grad_() for x in (q, k, v)]
        o, lse = ref_fp64.sparse_attention_fp64(*refs, ids, cu, max(lengths), block_size=b, scale=scale)
        o.backward(go.double())
        name = f"case{i}"
        for key, val in (("q", q), ("k", k), ("v", v), ("grad_out", go)):
            out[f"{name}/{key}"] = f32(val)
        out[f"{name}/indices"], out[f"{name}/cu"] = ids.numpy(), cu.numpy()
        out[f"{name}/out"], out[f"{name}/lse"] = f64(o), f64(lse)
        out[f"{name}/dq"], out[f"{name}/dk"], out[f"{name}/dv"] = (f64(x.grad) for x in refs)
        eo = eager.m3_sparse_attention(q, k, v, ids, cu, max(lengths), block_size=b, scale=scale)
        out[f"{name}/eager_out"] = f32(eo)
        meta.append(dict(name=name, lengths=lengths, groups=groups, ratio=ratio, dim=dim, block_size=b,
                         topk=topk, scale=scale))
    return out, meta


def gen_eager_error_cfg1(ref_fp64, eager):
    """Native BF16 eager error vs FP64 on configuration 1 (the fast path's tolerance yardstick)."""
    from msa_triton_b200.workloads import CONFIGS, make_inputs
    w = CONFIGS[1]
    x = make_inputs(w)
    cu = x["cu_seqlens"]
    with torch.no_grad():
        scores = eager.m3_index_score(x["index_q"], x["index_k"], cu, w.max_seqlen, block_size=w.block_size)
        ids = eager.m3_topk(scores, cu, block_size=w.block_size, topk_blocks=w.topk_blocks,
                            local_blocks=w.local_blocks)
    qkv = [x[n].clone().requires_grad_() for n in ("q", "k", "v")]
    o, lse = eager.m3_sparse_attention(*qkv, ids, cu, w.max_seqlen, block_size=w.block_size, return_lse=True)
    o.backward(x["grad_out"])
    refs = [x[n].double().requires_grad_() for n in ("q", "k", "v")]
    ro, rlse = ref_fp64.sparse_attention_fp64(*refs, ids, cu, w.max_seqlen, block_size=w.block_size)
    ro.backward(x["grad_out"].double())
    report = {}
    for nm, a, r in (("out", o, ro), ("lse", lse, rlse), ("dq", qkv[0].grad, refs[0].grad),
                     ("dk", qkv[1].grad, refs[1].grad), ("dv", qkv[2].grad, refs[2].grad)):
        a, r = a.detach().double(), r.detach()
        fin = torch.isfinite(r)
        err = (a[fin] - r[fin]).abs()
        # ref_rms: the float64 values' RMS, so that checks at other sizes can state the
        # max-abs error relative to the magnitude of what is being compared
        report[nm] = {"max_abs": float(err.max()), "rel_fro": float(err.norm() / r[fin].norm()),
                      "ref_rms": float(r[fin].square().mean().sqrt())}
    ids_np = ids.numpy()
    return report, ids_np, scores.numpy()


def gen_eager_numerics(eager):
    """The reference's native-dtype eager attention (outputs and gradients) on one packed bf16
    case: pins the oracle's restatement of its rounding points (sparse_attention_eager)."""
    from msa_triton_b200.workloads import random_selection
    gen = torch.Generator().manual_seed(3)
    lengths = [200, 0, 77]
    total = sum(lengths)
    q = torch.randn(total, 8, 32, generator=gen).bfloat16()
    k = torch.randn(total, 2, 32, generator=gen).bfloat16()
    v = torch.randn(total, 2, 32, generator=gen).bfloat16()
    go = torch.randn(total, 8, 32, generator=gen).bfloat16()
    ids = random_selection(lengths, 2, 32, 4, seed=2)
    cu = cu_of(lengths)
    qkv = [x.clone().requires_grad_() for x in (q, k, v)]
    out, lse = eager.m3_sparse_attention(*qkv, ids, cu, max(lengths), block_size=32, return_lse=True)
    out.backward(go)
    arrays = {"q": f32(q), "k": f32(k), "v": f32(v), "grad_out": f32(go), "indices": ids.numpy(), "cu": cu.numpy(),
              "out": f32(out), "lse": f32(lse), "dq": f32(qkv[0].grad), "dk": f32(qkv[1].grad),
              "dv": f32(qkv[2].grad)}
    return arrays, {"lengths": lengths, "block_size": 32, "max_seqlen": max(lengths), "dtype": "bf16"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--eager-error-only", action="store_true",
                    help="only recompute the configuration-1 eager error entry of the manifest")
    ap.add_argument("--eager-numerics-only", action="store_true",
                    help="only (re)write the eager-numerics fixture (eager.npz) and its manifest entry")
    args = ap.parse_args()
    eager, ref_fp64, ref_topk, ref_k2q = import_reference(args.reference)
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    if args.eager_numerics_only:
        manifest = json.loads((HERE / "manifest.json").read_text())
        arrays, meta = gen_eager_numerics(eager)
        np.savez_compressed(HERE / "eager.npz", **arrays)
        manifest["eager_numerics"] = meta
        (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
        return
    if args.eager_error_only:
        manifest = json.loads((HERE / "manifest.json").read_text())
        report, ids, _ = gen_eager_error_cfg1(ref_fp64, eager)
        old = np.load(HERE / "cfg1_selection.npz")["indices"]
        if not np.array_equal(old, ids):
            raise SystemExit("configuration-1 selection changed; regenerate every fixture")
        manifest["eager_error_cfg1"] = report
        print("eager error cfg1", report)
        (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
        return
    manifest = {}
    for stage, fn in (("score", lambda: gen_score(ref_fp64, eager)), ("topk", lambda: gen_topk(eager, ref_topk)),
                      ("k2q", lambda: gen_k2q(ref_k2q)), ("attention", lambda: gen_attention(ref_fp64, eager))):
        arrays, meta = fn()
        np.savez_compressed(HERE / f"{stage}.npz", **arrays)
        manifest[stage] = meta
        print(stage, len(meta), "cases")
    arrays, manifest["eager_numerics"] = gen_eager_numerics(eager)
    np.savez_compressed(HERE / "eager.npz", **arrays)
    report, ids, scores = gen_eager_error_cfg1(ref_fp64, eager)
    np.savez_compressed(HERE / "cfg1_selection.npz", indices=ids)
    manifest["eager_error_cfg1"] = report
    print("eager error cfg1", report)
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    main()
