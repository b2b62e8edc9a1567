"""Serving workload drivers (vramancer_b200.workloads) on CPU with tiny models: every
request finishes with its full output, speculation changes no greedy token, and the
prefill / decode drivers report positive rates."""
from vramancer_b200 import workloads


def _run(argv):
    args = workloads.parse_args(argv)
    info, dev, tp = workloads._init()
    fn = {"serve": workloads.run_serve, "spec": workloads.run_spec, "prefill": workloads.run_prefill,
          "decode": workloads.run_decode}[args.what]
    return fn(args, info, dev, tp)


def test_serve_finishes_every_request():
    r = _run(["serve", "--model", "tiny-qwen2", "--requests", "5", "--min-prompt", "8", "--max-prompt", "48",
              "--output", "6", "--kv-dtype", "fp8", "--prefill-chunk", "64"])
    assert r["output_tokens"] == 5 * 6
    assert r["output_tok_s"] > 0 and r["ttft_p50_ms"] > 0
    assert r["kv_dtype"] == "fp8"


def test_spec_keeps_greedy_tokens():
    r = _run(["spec", "--model", "tiny-qwen2", "--output", "20", "--batch", "2"])
    assert r["tokens_equal"] is True
    assert r["on"]["drafted"] >= r["on"]["accepted"] >= 0


def test_prefill_and_decode_drivers():
    r = _run(["prefill", "--model", "tiny-moe", "--batch", "2", "--seq", "32", "--iters", "1", "--warmup", "0"])
    assert r["prompt_tok_s"] > 0
    rows = _run(["decode", "--model", "tiny-gpt2", "--batches", "1,3", "--prompt-len", "12", "--steps", "3",
                 "--warmup", "1"])
    assert [x["batch"] for x in rows] == [1, 3] and all(x["tok_s"] > 0 for x in rows)


def test_cli_benchmark_workload(capsys):
    from vramancer_b200 import cli
    assert cli.main(["benchmark", "--workload", "decode", "--model", "tiny-qwen2", "--", "--batches", "2",
                     "--prompt-len", "8", "--steps", "2", "--warmup", "1"]) == 0
    out = capsys.readouterr().out
    assert '"workload": "decode"' in out and '"batch": 2' in out
