"""Regenerate the golden fixtures in tests/golden/ from the doerun/doe sources.

Run this in a container where the reference tree is mounted:

    python tests/golden/make_golden.py --reference /path/to/doe

It imports the reference's own numpy attention code
(``bench/tools/attention_kv_axis_sharded_stitch.py``: ``emit_local_partials``,
``shard_kv_along_position``, ``stitch_kv_axis_sharded_partials``) and its
canary test constants (``bench/tests/test_attention_canary_identity.py``),
and reads the attention-slice determinism fixtures
(``bench/fixtures/determinism/*attention-slice*``), and reads the ORT plugin
EP's session smoke cases as text
(``runtime/bridge/onnxruntime-ep/src/doe_ort_ep_session_smoke.cc``), copies
three of Doe's Gemma command streams (``examples/inference_gemma3_*``) and
hashes synthetic assets made by its generator
(``bench/lib/synthetic_assets.py``).  The outputs are small
.npz / .json files; nothing at test time reads the reference tree.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import re
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _import_reference(root: Path):
    sys.dont_write_bytecode = True  # the reference tree is read-only
    sys.path.insert(0, str(root))
    from bench.tools import attention_kv_axis_sharded_stitch as stitch_mod  # noqa: E402
    from bench.tests import test_attention_canary_identity as canary_mod  # noqa: E402
    return stitch_mod, canary_mod


def make_stitch_cases(stitch_mod) -> None:
    """Reference partials + stitch on random Q/K/V (the sharded-identity test's recipe)."""
    rng = np.random.default_rng(20261201)
    cases = {}
    idx = 0
    for head_dim in (8, 64, 128):
        for kv_len in (1, 3, 17, 40):
            for num_pes, slots in ((1, kv_len), (2, (kv_len + 1) // 2), (3, (kv_len + 2) // 3), (4, kv_len)):
                q = rng.standard_normal(head_dim).astype(np.float32)
                k = rng.standard_normal((kv_len, head_dim)).astype(np.float32)
                v = rng.standard_normal((kv_len, head_dim)).astype(np.float32)
                scale = np.float32(1.0 / np.sqrt(head_dim))
                ks, vs = stitch_mod.shard_kv_along_position(K=k, V=v, num_pes=num_pes, slots_per_pe=slots)
                partials = np.zeros((num_pes, head_dim + 2), np.float32)
                for pe in range(num_pes):
                    partials[pe] = stitch_mod.emit_local_partials(
                        Q=q, K_local=ks[pe], V_local=vs[pe], slot_base=pe * slots,
                        kv_len=kv_len, attn_scale=float(scale))
                out = stitch_mod.stitch_kv_axis_sharded_partials(partials)
                cases[f"c{idx}_q"] = q
                cases[f"c{idx}_k"] = k
                cases[f"c{idx}_v"] = v
                cases[f"c{idx}_meta"] = np.array([head_dim, kv_len, num_pes, slots], np.int64)
                cases[f"c{idx}_scale"] = np.array([scale], np.float32)
                cases[f"c{idx}_partials"] = partials
                cases[f"c{idx}_out"] = out
                idx += 1
    cases["count"] = np.array([idx], np.int64)
    np.savez_compressed(HERE / "stitch_reference.npz", **cases)


def make_canary(canary_mod) -> None:
    """Zero-input canary shas and the reference's own zero-input two-pass output."""
    shas = {str(k): v for k, v in canary_mod.CANARY_OUTPUT_SHAS.items()}
    checks = []
    for head_dim, kv_len in ((256, 15), (512, 7), (256, 1), (512, 4)):
        out = canary_mod._two_pass_attention_zero_input(head_dim=head_dim, kv_len=kv_len)
        checks.append({"head_dim": head_dim, "kv_len": kv_len,
                       "sha256": hashlib.sha256(out.tobytes()).hexdigest()})
    payload = {
        "source": "bench/tests/test_attention_canary_identity.py:41-48 (CANARY_OUTPUT_SHAS)",
        "canary_output_sha256": shas,
        "reference_zero_input_runs": checks,
    }
    (HERE / "canary.json").write_text(json.dumps(payload, indent=1) + "\n")


def make_slice_kat(root: Path) -> None:
    """Inputs and exact logits of the attention-slice determinism scenario."""
    det = root / "bench/fixtures/determinism"
    cmds = json.loads((det / "attention-slice-forward.commands.json").read_text())
    bufs = {c["handle"]: c["data"] for c in cmds if c["kind"] == "buffer_write"}
    out = {"source": "bench/fixtures/determinism/attention-slice-forward.commands.json; "
                     "{amd-vulkan,apple-metal}-attention-slice-logit-flip.json",
           "uniform_u32": bufs[4301], "q_u32": bufs[4302], "k_u32": bufs[4303],
           "v_u32": bufs[4304], "seq_len": 8, "head_dim": 8, "value_dim": 2}
    for name in ("amd-vulkan-attention-slice-logit-flip.json", "apple-metal-attention-slice-logit-flip.json"):
        meta = json.loads((det / name).read_text())
        out.setdefault("exact", {})[name] = {
            "exactReferenceLogits": meta["exactReferenceLogits"],
            "exactReferenceTopToken": meta["exactReferenceTopToken"],
        }
    (HERE / "attention_slice_kat.json").write_text(json.dumps(out, indent=1) + "\n")


def make_decode_sim(stitch_mod) -> None:
    """The decode simulator runner's inputs (default_rng(11); width 4, D 32, L 64).

    The expected output comes from the reference's single-shard partials +
    stitch (its two-pass body), the in-tree numpy path that runs here; the
    runner's own tolerance is atol 5e-5, rtol 5e-4
    (bench/runners/csl-runners/attention_decode_sim_runner.py:45-48, 88).
    """
    width, head_dim, kv_len, q_len = 4, 32, 64, 1
    scale = np.float32(0.125)
    rng = np.random.default_rng(seed=11)
    q = rng.standard_normal(size=(width, q_len, head_dim), dtype=np.float32)
    k = rng.standard_normal(size=(width, kv_len, head_dim), dtype=np.float32)
    v = rng.standard_normal(size=(width, kv_len, head_dim), dtype=np.float32)
    expected = np.zeros((width, head_dim), np.float32)
    for pe in range(width):
        part = stitch_mod.emit_local_partials(Q=q[pe, 0], K_local=k[pe], V_local=v[pe], slot_base=0,
                                              kv_len=kv_len, attn_scale=float(scale))
        expected[pe] = stitch_mod.stitch_kv_axis_sharded_partials(part[None, :])
    np.savez_compressed(HERE / "decode_sim_seed11.npz", q=q, k=k, v=v, scale=np.array([scale]),
                        expected=expected, tol=np.array([5e-5, 5e-4]))


def _braced(text: str, start: int) -> str:
    """The balanced {...} group that opens at or after text[start]."""
    i = text.index("{", start)
    depth = 0
    for j in range(i, len(text)):
        depth += {"{": 1, "}": -1}.get(text[j], 0)
        if depth == 0:
            return text[i:j + 1]
    raise ValueError("unbalanced braces")


def _numbers(group: str) -> list:
    """Nested numeric initialiser lists ({1.0f, -2.0f} / {{1, 4}, {4}}) as lists."""
    inner = group.strip()[1:-1].strip()
    if inner.startswith("{"):
        out, pos = [], 0
        while True:
            k = inner.find("{", pos)
            if k < 0:
                return out
            g = _braced(inner, k)
            out.append(_numbers(g))
            pos = k + len(g)
    return [float(t.rstrip("f")) for t in re.findall(r"-?\d+(?:\.\d*)?(?:e-?\d+)?f?", inner)]


def make_ort_ep_cases(root: Path) -> None:
    """The ORT plugin EP's session smoke cases (inputs and expected outputs)."""
    src = (root / "runtime/bridge/onnxruntime-ep/src/doe_ort_ep_session_smoke.cc").read_text()
    body = _braced(src, src.index("std::vector<SmokeCaseSpec> BuildSmokeCases()"))
    cases, pos = [], 0
    while True:
        k = body.find("SmokeCaseSpec{", pos)
        if k < 0:
            break
        spec = _braced(body, k)
        pos = k + len(spec)
        name = re.search(r'\.case_name = "([a-z_]+)"', spec).group(1)
        field = lambda f: _numbers(_braced(spec, spec.index(f".{f} =")))
        cases.append({"name": name, "input_dims": [[int(d) for d in dims] for dims in field("input_dims")],
                      "output_dims": [int(d) for d in field("output_dims")],
                      "inputs": field("inputs"), "expected": field("expected_output")})
    out = {"source": "runtime/bridge/onnxruntime-ep/src/doe_ort_ep_session_smoke.cc:808-950 (BuildSmokeCases); "
                     "tolerance :578-584 (absolute 1e-5)",
           "tolerance_abs": 1e-5, "cases": cases}
    (HERE / "ort_ep_smoke_cases.json").write_text(json.dumps(out, indent=1) + "\n")


GEMMA_STREAMS = ("inference_gemma3_270m_decode_1tok_commands", "inference_gemma3_1b_decode_1tok_commands",
                 "inference_gemma3_270m_prefill_32tok_commands")


def make_command_streams(root: Path) -> None:
    """Doe's Gemma command streams (examples/<name>.json, the reference's own
    replay inputs), re-serialised compactly, and the sha256 of the synthetic
    asset of every buffer_load of the 270m decode stream plus a few small
    cases, computed by the reference's generator
    (bench/lib/synthetic_assets.py:generate_asset_bytes)."""
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(root))
    from bench.lib import synthetic_assets as sa  # noqa: E402

    streams = {}
    for name in GEMMA_STREAMS:
        streams[name] = json.loads((root / "examples" / f"{name}.json").read_text())
    (HERE / "gemma_command_streams.json").write_text(
        json.dumps({"source": "examples/<name>.json of the doerun/doe tree", "streams": streams},
                   separators=(",", ":")) + "\n")
    cases = []
    for gen, seed, scale, n in (("splitmix64_f32_nonzero_v1", 0, 1.0, 64), ("splitmix64_f32_nonzero_v1", 7, 0.125, 4096),
                                ("splitmix64_f32_nonzero_v1", 2 ** 63 + 5, 3.5, 1024),
                                ("splitmix64_f16_nonzero_v1", 11, 0.5, 2048),
                                ("splitmix64_f32_nonzero_v1", 123, 1e-7, 256)):
        data = sa.generate_asset_bytes(generator=gen, seed=seed, scale=scale, byte_length=n)
        cases.append({"generator": gen, "seed": seed, "scale": scale, "byteLength": n,
                      "sha256": hashlib.sha256(data).hexdigest(), "head_hex": data[:32].hex()})
    stream_assets = []
    for c in streams["inference_gemma3_270m_decode_1tok_commands"]:
        if c["kind"] != "buffer_load":
            continue
        data = sa.generate_asset_bytes(generator=c["generator"], seed=c["seed"], scale=c["scale"],
                                       byte_length=c["byteLength"])
        stream_assets.append({"handle": c["handle"], "sha256": hashlib.sha256(data).hexdigest()})
    (HERE / "synthetic_assets.json").write_text(json.dumps(
        {"source": "bench/lib/synthetic_assets.py:generate_asset_bytes (splitmix64 nonzero generators)",
         "cases": cases, "inference_gemma3_270m_decode_1tok": stream_assets}, indent=1) + "\n")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    ap.add_argument("--only", choices=["stitch", "canary", "slice", "decode_sim", "ort_ep", "streams"], default=None,
                    help="regenerate one fixture only")
    args = ap.parse_args()
    if args.only == "ort_ep":
        make_ort_ep_cases(args.reference)
        print("golden fixtures written to", HERE)
        return
    if args.only == "streams":
        make_command_streams(args.reference)
        print("golden fixtures written to", HERE)
        return
    stitch_mod, canary_mod = _import_reference(args.reference)
    if args.only in (None, "stitch"):
        make_stitch_cases(stitch_mod)
    if args.only in (None, "canary"):
        make_canary(canary_mod)
    if args.only in (None, "slice"):
        make_slice_kat(args.reference)
    if args.only in (None, "decode_sim"):
        make_decode_sim(stitch_mod)
    if args.only is None:
        make_ort_ep_cases(args.reference)
        make_command_streams(args.reference)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
