"""Regenerate the committed golden fixtures (run in a container that has the
reference checkout; the fixtures themselves travel, the reference does not).

    python tests/golden/make_golden.py --reference <path of the reference checkout>
    python tests/golden/make_golden.py --greedy | --batched   (need only oracle/_ref)

Writes
  tests/golden/ame_cases.npz   the 12 shipped AME cases of
      rtl_verification/cases/*: inputs (a.bin or a_src.bin, b.bin, strides),
      expected c_ref.bin / c_peak.bin words and xor_ref (mixed cases).
  tests/golden/greedy_ref.npz   BASELINE config 3 (seed-0 random-init model,
      32-token seeded prompt, 64 greedy steps) run by the reference's own
      qwen3.c + kernels_scalar.c / kernels_hwsim.c (oracle/_ref): generated
      tokens and each step's top-8 logits (ids, values).
  tests/golden/config1_exact.npz   BASELINE config 1 (16x1024x2048, seed 0,
      this project's seeded generator) evaluated by the reference's own
      generator function ame_gemm_ref (40_gen_ame_vectors.py:121-143), imported
      from the reference checkout with K_BLOCK set to 16 and to 32.
  tests/golden/batched_ref.npz   rows of the two benched batches (bench.py's
      configs[3] prefill and configs[4] decode inputs) run by the reference's
      own qwen3.c + kernels_scalar.c (oracle/_ref) in 128-token calls: top-64
      logits, the logits at every 37th id and max|logit| of each output row,
      and the greedy ids.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import multiprocessing as mp
import os
import struct
import sys
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))

CONFIG1 = dict(M=16, K=1024, N=2048, seed=0, a_stream=0x41, b_stream=0x42,
               a_sigma=1.0, b_sigma=0.02)


def words(path: Path, dtype):
    data = path.read_bytes()
    return np.frombuffer(data, dtype=dtype).copy()


def load_cases(ref: Path):
    root = ref / "rtl_verification" / "cases"
    out = {}
    names = []
    for d in sorted(root.iterdir()):
        meta = json.loads((d / "meta.json").read_text(encoding="utf-8"))
        cid = meta["case_id"]
        M, N, K = meta["shape"]["M"], meta["shape"]["N"], meta["shape"]["K"]
        sa = meta["stride_bytes"]["a"]
        sb = meta["stride_bytes"]["b"]
        mixed = bool(meta.get("mixed"))
        names.append(cid)
        if mixed:
            # a_src is FP32 laid out on the BF16 A's element stride
            a_src = words(d / "a_src.bin", np.float32).reshape(M, sa // 2)
            out[f"{cid}/a_src"] = a_src
            lda = sa // 2
        else:
            a = words(d / "a.bin", np.uint16).reshape(M, sa // 2)
            out[f"{cid}/a"] = a
            lda = sa // 2
        b = words(d / "b.bin", np.uint16).reshape(N, sb // 2)
        out[f"{cid}/b"] = b
        out[f"{cid}/c_ref"] = words(d / "c_ref.bin", np.uint32).reshape(M, N)
        out[f"{cid}/c_peak"] = words(d / "c_peak.bin", np.float32).reshape(M, N)
        if (d / "xor_ref.bin").exists():
            out[f"{cid}/xor_ref"] = words(d / "xor_ref.bin", np.uint32)
        out[f"{cid}/shape"] = np.array([M, N, K, lda, sb // 2, int(mixed)], np.int64)
    out["case_ids"] = np.array(names)
    return out


def _import_generator(ref: Path):
    path = ref / "rtl_verification" / "golden_src" / "40_gen_ame_vectors.py"
    spec = importlib.util.spec_from_file_location("ame_gen_ref", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


_GEN = None


def _rows(args):
    ref, kblock, A_rows, B = args
    global _GEN
    if _GEN is None:
        _GEN = _import_generator(Path(ref))
    _GEN.K_BLOCK = kblock
    C = _GEN.ame_gemm_ref(A_rows, B, len(A_rows), len(B), len(B[0]))
    return C


def config1(ref: Path):
    import oracle
    c = CONFIG1
    A = oracle.synth_normal_bf16((c["M"], c["K"]), c["seed"], c["a_stream"], c["a_sigma"])
    B = oracle.synth_normal_bf16((c["N"], c["K"]), c["seed"], c["b_stream"], c["b_sigma"])
    Al, Bl = A.tolist(), B.tolist()
    res = {}
    with mp.get_context("spawn").Pool() as pool:
        for kb in (16, 32):
            jobs = [(str(ref), kb, [Al[m]], Bl) for m in range(c["M"])]
            rows = pool.map(_rows, jobs)
            res[f"c_kb{kb}"] = np.array([r[0] for r in rows], np.uint32)
    # Inputs are regenerated from the seed by the tests; only their digests
    # are kept, so generator drift is caught without committing 4 MB.
    res["a_sha256"] = np.frombuffer(hashlib.sha256(A.tobytes()).digest(), np.uint8)
    res["b_sha256"] = np.frombuffer(hashlib.sha256(B.tobytes()).digest(), np.uint8)
    res["meta"] = np.array([c["M"], c["K"], c["N"], c["seed"]], np.int64)
    return res


PROMPT = dict(seed=0, stream=0x544F4B, n=32, steps=64)


def greedy_reference():
    import oracle
    blob = oracle.qw3m_blob(seed=0, sigma=0.02)
    prompt = oracle.synth_tokens(PROMPT["n"], PROMPT["seed"], PROMPT["stream"])
    res = {"prompt": prompt}
    for kern in ("scalar", "hwsim"):
        m = oracle.RefModel(blob, kern)
        toks, top_i, top_v = [], [], []
        logits = m.forward_batch(prompt, 0)
        pos = PROMPT["n"]
        for step in range(PROMPT["steps"]):
            order = np.argsort(-logits, kind="stable")[:8]
            top_i.append(order.astype(np.int32))
            top_v.append(logits[order].astype(np.float32))
            nxt = int(oracle.argmax(logits))
            toks.append(nxt)
            if step + 1 < PROMPT["steps"]:
                logits = m.forward_batch(np.array([nxt], np.int32), pos)
                pos += 1
        res[f"{kern}_tokens"] = np.array(toks, np.int32)
        res[f"{kern}_top_ids"] = np.stack(top_i)
        res[f"{kern}_top_vals"] = np.stack(top_v)
        print(kern, toks[:16])
    return res


# Benched batches (bench.py): configs[3] prefill = synth_tokens(64 * 512, 0,
# TOKEN_STREAM) as 64 rows of 512; configs[4] decode context =
# synth_tokens(256 * 1024, 1, TOKEN_STREAM) as 256 rows of 1024. The fixtures
# hold the reference's logits for the first and the last row of each batch.
TOKEN_STREAM = 0x544F4B
CHUNK = 128                       # QWEN3_MAX_BATCH: tokens per qwen3_forward_batch call
SAMPLE_STRIDE = 37                # logits kept at ids 0, 37, 74, ... (4107 of 151936)
TOP = 64


def _logit_summary(logits):
    """Top-64 ids/values, the values at every 37th id and max|logit| of one row."""
    order = np.argsort(-logits, kind="stable")[:TOP]
    return (order.astype(np.int32), logits[order].astype(np.float32),
            logits[::SAMPLE_STRIDE].astype(np.float32), np.float32(np.abs(logits).max()))


def _batched_worker(job):
    """One spawned process: the reference's own qwen3.c + kernels_scalar.c +
    ops_scalar.c (oracle/_ref) on one row of a benched batch, prefilled in
    128-token qwen3_forward_batch calls (the reference caps a call at
    QWEN3_MAX_BATCH = 128, qwen3.c:461), then `steps` greedy single-token calls."""
    kind, row, seqs, length, seed, steps = job
    import oracle
    blob = oracle.qw3m_blob(seed=0, sigma=0.02)
    m = oracle.RefModel(blob, "scalar")
    toks = oracle.synth_tokens(seqs * length, seed, TOKEN_STREAM)[row * length:(row + 1) * length]
    for p0 in range(0, length, CHUNK):
        logits = m.forward_batch(toks[p0:p0 + CHUNK], p0)
    out = [_logit_summary(logits)]
    chosen = [oracle.argmax(logits)]
    pos = length
    for _ in range(steps):
        logits = m.forward_batch(np.array([chosen[-1]], np.int32), pos)
        pos += 1
        out.append(_logit_summary(logits))
        chosen.append(oracle.argmax(logits))
    print(kind, row, "done", chosen, flush=True)
    return kind, row, out, chosen


def batched_reference():
    """configs[3] rows 0 and 63 (512-token prefill: last-token logits) and
    configs[4] rows 0 and 255 (1024-token context: the prefill's last-token
    logits, then 8 greedy steps at positions 1024-1031, 9 logit rows each)."""
    jobs = [("c4", 0, 64, 512, 0, 0), ("c4", 63, 64, 512, 0, 0),
            ("c5", 0, 256, 1024, 1, 8), ("c5", 255, 256, 1024, 1, 8)]
    with mp.get_context("spawn").Pool(len(jobs)) as pool:
        res = pool.map(_batched_worker, jobs)
    out = {"sample_stride": np.int32(SAMPLE_STRIDE), "chunk": np.int32(CHUNK)}
    for kind, rows in (("c4", (0, 63)), ("c5", (0, 255))):
        got = {r[1]: r for r in res if r[0] == kind}
        out[f"{kind}_rows"] = np.array(rows, np.int32)
        for name, i in (("top_ids", 0), ("top_vals", 1), ("sampled", 2), ("absmax", 3)):
            out[f"{kind}_{name}"] = np.stack([np.stack([s[i] for s in got[r][2]]) for r in rows])
        out[f"{kind}_tokens"] = np.array([got[r][3] for r in rows], np.int32)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("N550_REFERENCE"),
                    help="reference checkout (default: $N550_REFERENCE)")
    ap.add_argument("--skip-config1", action="store_true")
    ap.add_argument("--greedy", action="store_true", help="only the greedy-decode fixture")
    ap.add_argument("--batched", action="store_true",
                    help="only the benched-batch fixture (batched_ref.npz)")
    args = ap.parse_args()
    here = Path(__file__).resolve().parent
    if args.greedy:
        np.savez_compressed(here / "greedy_ref.npz", **greedy_reference())
        print("wrote greedy_ref.npz")
        return
    if args.batched:
        np.savez_compressed(here / "batched_ref.npz", **batched_reference())
        print("wrote batched_ref.npz")
        return
    if not args.reference:
        ap.error("--reference (or N550_REFERENCE) is required for the AME cases")
    ref = Path(args.reference)
    cases = load_cases(ref)
    np.savez_compressed(here / "ame_cases.npz", **cases)
    print("wrote ame_cases.npz:", list(cases["case_ids"]))
    if not args.skip_config1:
        res = config1(ref)
        np.savez_compressed(here / "config1_exact.npz", **res)
        print("wrote config1_exact.npz")


if __name__ == "__main__":
    main()
