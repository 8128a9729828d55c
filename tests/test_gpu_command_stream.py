"""GPU: Doe's Gemma command streams replayed on the CUDA backend through
doe_cuda_dispatch (doe_b200/command_stream.py), every kernel_dispatch a
kernel of libdoe_cuda.so.

Streams (tests/golden/gemma_command_streams.json, copies of the reference's
examples/inference_gemma3_*_commands.json): Gemma 3 270M and 1B one-token
decode (rmsnorm, matmul-gemv, rope, attention-decode, residual, gelu,
sample) and Gemma 3 270M 32-token prefill (gather, rmsnorm, matmul-tiled,
rope, attention-prefill, residual, gelu).

- Stage by stage: after each dispatch the written buffer is captured and
  compared with the CPU restatement of that WGSL kernel (oracle/pipeline.py)
  fed the GPU's own inputs, within 1e-5 * max(|ref|, 1) (the f32 bar);
  rope and gather are bit-exact, sample's token equal.
- End to end: the decode streams' sampled token equals the token of the
  whole stream replayed on the CPU oracle.
"""
from __future__ import annotations

import json

import numpy as np
import pytest

from doe_b200 import command_stream as cs
from oracle import pipeline as opl
from tests.gpu_util import within

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

STREAMS = ("inference_gemma3_270m_decode_1tok_commands", "inference_gemma3_1b_decode_1tok_commands",
           "inference_gemma3_270m_prefill_32tok_commands")
EXACT = {"rope.wgsl", "gather.wgsl", "residual.wgsl"}


@pytest.fixture(scope="module")
def streams(golden_dir):
    return json.loads((golden_dir / "gemma_command_streams.json").read_text())["streams"]


@pytest.mark.parametrize("name", STREAMS)
def test_stream_stage_by_stage_and_end_to_end(name, streams):
    cmds = streams[name]
    r = cs.Replayer()
    mirror: dict[int, bytes] = {}
    seen = []
    try:
        for c in cmds:
            r.execute(c)
            if c["kind"] != "kernel_dispatch":
                mirror[int(c["handle"])] = r.payload(c)
                continue
            binds = {int(b["binding"]): (int(b["resource_handle"]), int(b["buffer_size"])) for b in c["bindings"]}
            h, ref = opl.run_dispatch(c["kernel"], c.get("entry_point"), int(c.get("x", 1)), mirror, binds)
            size = next(sz for hh, sz in binds.values() if hh == h)
            got_raw = r.capture(h, size)
            ref = np.asarray(ref)
            got = np.frombuffer(got_raw[:ref.nbytes], ref.dtype)
            if c["kernel"] == "sample.wgsl" or c["kernel"] in EXACT:
                assert np.array_equal(got, ref), (c["kernel"], len(seen))
            else:
                within(got, ref, 1e-5)
            prev = mirror.get(h, b"\0" * size).ljust(size, b"\0")
            mirror[h] = got_raw[:ref.nbytes] + prev[ref.nbytes:]
            seen.append(c["kernel"])
        r.backend.flush_queue()
    finally:
        r.backend.close()
    assert len(seen) == sum(1 for c in cmds if c["kind"] == "kernel_dispatch")
    if seen[-1] == "sample.wgsl":
        _, log = opl.replay(cmds, cs.synthetic_asset)
        cpu_token = int(np.frombuffer(log[-1][2], np.uint32)[0])
        gpu_token = int(np.frombuffer(mirror[log[-1][1]][:4], np.uint32)[0])
        assert gpu_token == cpu_token
