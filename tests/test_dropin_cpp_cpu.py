"""The C++ drop-in on CPU: a caller written against the reference's C++ API
(tests/cpp/reference_style_caller.cc: Tokenizer, OlmoeModel::Load's failure
path, RoutingTrace I/O, LruPolicy / OsPageCachePolicy / LearnedPinPolicy,
Replay, BuildUsage, SweepBudgets) compiles against include/nuthatch/ with
g++, links libnuthatch_b200.so, runs, and prints what the Python mirror of
the same calls gives."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

import nuthatch_b200 as nh
from nuthatch_b200._lib import LIB_PATH

ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_reference_style_cpp_caller_links_and_agrees(tmp_path):
    import gguf

    tok_path = tmp_path / "tok.gguf"
    w = gguf.GGUFWriter(str(tok_path), "olmoe")
    vocab = ["h", "e", "l", "o", "Ġ", "w", "r", "d", "he", "ll", "hell", "hello", "Ġw", "or", "Ġwor", "Ġworl",
             "Ġworld"]
    w.add_token_list(vocab)
    w.add_token_merges(["h e", "l l", "he ll", "hell o", "Ġ w", "o r", "Ġw or", "Ġwor l", "Ġworl d"])
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()

    exe = tmp_path / "caller"
    lib_dir = Path(LIB_PATH).parent
    subprocess.run(["g++", "-std=c++17", "-Wall", "-Werror", f"-I{ROOT / 'include'}",
                    str(ROOT / "tests" / "cpp" / "reference_style_caller.cc"), f"-L{lib_dir}", "-lnuthatch_b200",
                    f"-Wl,-rpath,{lib_dir}", "-o", str(exe)], check=True, timeout=300)
    trace_path = tmp_path / "trace.bin"
    run = subprocess.run([str(exe), str(tok_path), str(trace_path), "hello", "world"], capture_output=True,
                         text=True, timeout=60)
    assert run.returncode == 0, run.stderr
    lines = run.stdout.splitlines()

    tk = nh.Tokenizer.Load(str(tok_path))
    ids = tk.Encode("hello world")
    assert lines[0] == f"vocab {len(vocab)}"
    assert lines[1] == "ids " + " ".join(map(str, ids)) and ids == [11, 16]
    assert lines[2] == "text hello world"
    assert lines[3] == "model null"

    back = nh.RoutingTrace()
    assert nh.ReadRoutingTrace(str(trace_path), back) and len(back.records) == 36
    usage = nh.BuildUsage(back, 8)
    hits = [nh.Replay(back, p).hits for p in (nh.LruPolicy(3, 3), nh.OsPageCachePolicy(9),
                                              nh.LearnedPinPolicy(3, 2, 1, usage))]
    assert lines[4] == f"replay {hits[0]} {hits[1]} {hits[2]} of 108"
    rows = nh.SweepBudgets(back, [2, 4])
    assert lines[5:7] == [f"sweep {b} {l:.6f} {r:.6f} {o:.6f}" for b, l, r, o in rows]
