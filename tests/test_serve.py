"""Host logic of the kernel-folder binary (serve.py): flags and --serve request validation, with
the reference's messages (LK/main.swift:513-524)."""

import json

import pytest

from gemmagemini4hackathon2026_10_2425_b200 import serve


def test_flags_of_the_reference_binary():
    a = serve.parse_args(["--weights", "w.bin", "--serve", "--max-ctx", "128", "--no-gemm", "--define", "X=1"])
    assert a.weights == "w.bin" and a.serve and a.max_ctx == 128
    a = serve.parse_args(["--weights", "w.bin", "--prompt-ids", "1,2,3", "--gen", "4", "--dump-logits", "l.bin"])
    assert a.prompt_ids == "1,2,3" and a.gen == 4 and a.dump_logits == "l.bin"
    a = serve.parse_args(["--weights", "w.bin", "--bench-pp", "512", "--bench-tg", "128", "--reps", "3"])
    assert (a.bench_pp, a.bench_tg, a.reps) == (512, 128, 3)


def test_request_ok_and_clamped():
    ids, mt, stop = serve.parse_request(json.dumps({"ids": [1, 2, 3], "max_tokens": 100, "stop_ids": [7, 9]}), 256, 64)
    assert ids == [1, 2, 3] and mt == 61 and stop == {7, 9}
    ids, mt, stop = serve.parse_request('{"ids": [5]}', 256, 4096)
    assert mt == 256 and stop == set()


@pytest.mark.parametrize(
    "line,msg",
    [
        ("not json", "expected"),
        ('{"max_tokens": 3}', "expected"),
        ('{"ids": []}', "expected"),
        ('{"ids": [1, 300]}', "token id 300 out of range"),
        ('{"ids": [-1]}', "token id -1 out of range"),
        (json.dumps({"ids": list(range(64))}), "prompt has 64 tokens, max_ctx is 64"),
    ],
)
def test_bad_requests(line, msg):
    with pytest.raises(ValueError, match=msg):
        serve.parse_request(line, 256, 64)
