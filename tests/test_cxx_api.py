"""The reference's C++ interfaces as this library exports them (include/g4dense/runner.hpp,
draft_runtime.hpp, speculator.hpp, sampling.hpp, device_context.hpp): a C++ program compiled
against the public headers and linked with libg4dense_b200.so, as the reference's own C++
callers (src/main.cpp, src/server.cpp, its tests) use ForwardRunner, DraftRuntime and
SpeculativeCoordinator. Reference: include/g4dense/runner.hpp:100-157, draft_runtime.hpp:19-54,
speculator.hpp:24-31.

CPU: the known answers of the reference's sampling and speculative tests through the C++ API, and
the container validators (csrc/format.cpp) on hand-made headers. GPU: ForwardRunner's batched
and single-token passes, greedy speculative generate_tokens (tokens and round records) and
DraftRuntime drafting, each against the CPU oracle."""
from __future__ import annotations

import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

REPO = Path(__file__).resolve().parents[1]
CPP = Path(__file__).resolve().parent / "cpp"


@pytest.fixture(scope="module")
def cxx_test_bin(built_lib, tmp_path_factory):
    out = tmp_path_factory.mktemp("cxx") / "test_cxx_api"
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(REPO / "include"), str(CPP / "test_cxx_api.cpp"),
                        "-o", str(out), str(built_lib), f"-Wl,-rpath,{built_lib.parent}"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    return out


def test_cxx_api_known_answers(cxx_test_bin):
    r = subprocess.run([str(cxx_test_bin), "cpu"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_format_validators(tmp_path):
    out = tmp_path / "test_format"
    csrc = REPO / "turbo-winfare-dense_b200" / "csrc"
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(csrc), str(CPP / "test_format.cpp"),
                        str(csrc / "format.cpp"), "-o", str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    r = subprocess.run([str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


def test_tensor_parallel_shard_plan(tmp_path):
    """The engine's split of each layer across tp = 1, 2, 4, 8 ranks (csrc/shard.h), on the host."""
    out = tmp_path / "test_shard"
    csrc = REPO / "turbo-winfare-dense_b200" / "csrc"
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-I", str(csrc), str(CPP / "test_shard.cpp"), "-o", str(out)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    r = subprocess.run([str(out)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.gpu
def test_cxx_runner_drafter_speculator_match_oracle(cxx_test_bin, config0):
    from g4dense_b200 import container as C
    tgt, drf = config0["target_centered"], config0["draft_centered"]
    prompt = C.pinned_prompt()
    n = C.PINNED_TOKENS
    r = subprocess.run([str(cxx_test_bin), "gpu", str(tgt), str(drf), ",".join(str(int(t)) for t in prompt), str(n)],
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr[-3000:]
    got = json.loads(r.stdout.strip().splitlines()[-1])
    T = O.RestatedModel(tgt)
    want_am = [int(np.argmax(T.forward(int(t), p))) for p, t in enumerate(prompt[:8])]
    assert got["argmax_batched"] == want_am and got["argmax_single"] == want_am
    assert got["batched_vs_single_max_diff"] < 1e-2
    plain, _ = O.spec_generate(O.RestatedModel(tgt), None, prompt, n)
    spec, rounds = O.spec_generate(O.RestatedModel(tgt), O.RestatedModel(drf), prompt, n, verify_width=5)
    assert got["plain"] == plain.tolist()
    assert got["spec"] == spec.tolist() and got["spec_streamed"] == len(spec)
    assert got["rounds"] == [list(x) for x in rounds]
    # DraftRuntime: the drafter's greedy continuation, teacher-forced on the oracle.
    D = O.RestatedModel(drf)
    ctx = [int(t) for t in prompt]
    for p, t in enumerate(ctx[:-1]):
        D.forward(t, p)
    want, cur, pos = [], ctx[-1], len(ctx) - 1
    for _ in range(4):
        cur = int(np.argmax(D.forward(cur, pos)))
        want.append(cur)
        pos += 1
    assert got["draft1"] == want
    D.truncate(len(ctx) + 1)  # kept: prompt + 2 drafts; the second kept draft is not yet forwarded
    want2, cur, pos = [], want[1], len(ctx) + 1
    for _ in range(3):
        cur = int(np.argmax(D.forward(cur, pos)))
        want2.append(cur)
        pos += 1
    assert got["draft2"] == want2


@pytest.fixture(scope="module")
def tok_api_bin(built_lib, tmp_path_factory):
    out = tmp_path_factory.mktemp("cxxtok") / "test_tokenizer_api"
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-I", str(REPO / "include"), str(CPP / "test_tokenizer_api.cpp"),
                        "-o", str(out), str(built_lib), f"-Wl,-rpath,{built_lib.parent}"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    return out


def test_cxx_tokenizer_api(tok_api_bin, tmp_path):
    """Tokenizer / IncrementalDetokenizer / StreamingStopMatcher through the public C++ headers,
    with the reference's own test cases (tests/test_tokenizer.cpp, tests/test_detokenizer.cpp)."""
    r = subprocess.run([str(tok_api_bin), "cpu", str(tmp_path)], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.gpu
def test_cxx_runner_text_generate(tok_api_bin, config0, tmp_path):
    """ForwardRunner::generate(prompt) with a tokenizer: greedy, chat template, stop ids; tokens and
    pieces equal the reference tokenizer + restated runner on the same container."""
    from g4dense_b200 import synth_tokenizer as S
    from oracle import tokenizer_oracle as TO
    tokp = S.write_synthetic_tokenizer(tmp_path / "tokenizer.json")
    prompt = S.STOP_PROMPT
    R = O.ReferenceTokenizer(tokp) if O.reference_available() else TO.Tokenizer(tokp)
    tgt = config0["target_centered"]
    ids = R.encode(R.chat_template([("user", prompt)]), False)
    want, _ = O.spec_generate(O.RestatedModel(tgt), None, ids, 48)
    want = want.tolist()
    stops = R.stop_ids() if callable(R.stop_ids) else R.stop_ids
    cut = next(i for i, t in enumerate(want) if t in stops)
    want = want[:cut + 1]
    r = subprocess.run([str(tok_api_bin), "gpu", str(tgt), str(tokp), prompt, "48"], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr[-3000:]
    got = json.loads(r.stdout.strip().splitlines()[-1])
    assert got["tokens"] == want
    assert [bytes.fromhex(p) for p in got["pieces"]] == [R.decode_single(t) for t in want]
