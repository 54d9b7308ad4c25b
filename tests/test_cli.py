"""CLI parsing and CPU end-to-end subcommands (reference src/bin/air_rs.rs:729-804 parser tests)."""
import pytest

from air_rs.cli import build_parser, main
from air_rs.gguf import GGMLType
from air_rs.models.config import tiny_llama
from air_rs.models.random_init import write_random_gguf


def test_generate_defaults():
    a = build_parser().parse_args(["generate", "-m", "m.gguf", "-p", "hi"])
    assert (a.max_tokens, a.temperature, a.top_p, a.tp, a.draft_max, a.epsilon) == (512, 0.7, 0.9, 1, 5, 0.15)
    assert not a.stream and a.model_draft is None


def test_serve_defaults_and_aliases():
    a = build_parser().parse_args(["serve", "-m", "m.gguf"])
    assert (a.port, a.host, a.reasoning_format, a.guided_decoding_backend) == (8080, "127.0.0.1", "auto", "xgrammar")
    a = build_parser().parse_args(["serve", "-m", "m.gguf", "-P", "9000", "--max-batch-size", "7"])
    assert a.port == 9000 and a.max_num_seqs == 7


def test_bench_defaults():
    a = build_parser().parse_args(["bench", "-m", "m.gguf"])
    assert (a.n_tokens, a.runs) == (512, 3)


def test_tls_pair_required(tmp_path):
    assert main(["serve", "-m", "x.gguf", "--tls-cert", "c.pem"]) == 2


def test_missing_required():
    with pytest.raises(SystemExit):
        build_parser().parse_args(["generate", "-m", "m.gguf"])


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    p = tmp_path_factory.mktemp("c") / "tiny.gguf"
    return write_random_gguf(str(p), tiny_llama(), GGMLType.Q8_0)


def test_info_and_generate_cpu(tiny, capsys):
    assert main(["info", "-m", tiny]) == 0
    out = capsys.readouterr().out
    assert "2 layers, hidden 256, heads 4/2" in out
    assert main(["generate", "-m", tiny, "-p", "hello", "-n", "4", "-t", "0", "--device", "cpu"]) == 0
    assert main(["--run", tiny, "hey", "-n", "3", "--device", "cpu"]) == 0
