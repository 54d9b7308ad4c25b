"""Public Python API (ported from the reference's python/tests/test_bindings.py tiers 1-2,
plus the tier-3 model tests run against a tiny random GGUF on the CPU oracle path)."""
import asyncio
import inspect

import pytest
import torch

import air_rs
from air_rs import GenerateConfig, GbnfConstraint, utils
from air_rs.gguf import GGMLType
from air_rs.models.config import tiny_llama
from air_rs.models.random_init import write_random_gguf


class TestUtils:
    def test_chatml_basic(self):
        p = utils.format_chat([{"role": "user", "content": "hi"}], "chatml")
        assert p == "<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"

    def test_llama3_bos(self):
        assert utils.format_chat([{"role": "user", "content": "x"}], "llama3").startswith("<|begin_of_text|>")

    def test_mistral_system_prepended(self):
        p = utils.format_chat([{"role": "system", "content": "S"}, {"role": "user", "content": "U"}], "mistral")
        assert "[INST] S\n\nU [/INST]" in p

    def test_no_generation_prompt(self):
        p = utils.format_chat([{"role": "user", "content": "x"}], "chatml", add_generation_prompt=False)
        assert not p.endswith("assistant\n")

    def test_unknown_template_raises(self):
        with pytest.raises(ValueError):
            utils.format_chat([], "nope")

    def test_phi3_and_gemma(self):
        assert "<|user|>\nq<|end|>" in utils.format_chat([{"role": "user", "content": "q"}], "phi3")
        assert "<start_of_turn>user\nq<end_of_turn>" in utils.format_chat([{"role": "user", "content": "q"}], "gemma")

    def test_count_tokens_approx(self):
        assert utils.count_tokens_approx("") == 1
        assert utils.count_tokens_approx("a" * 40) == 10


class TestTypes:
    def test_version_string(self):
        assert isinstance(air_rs.__version__, str) and air_rs.__version__.count(".") == 2

    def test_generate_config_defaults(self):
        c = GenerateConfig()
        assert (c.max_tokens, c.temperature, c.top_p, c.top_k, c.repetition_penalty) == (512, 0.7, 0.9, 40, 1.1)
        assert c.stop_strings == [] and c.grammar is None

    def test_generate_config_custom(self):
        c = GenerateConfig(max_tokens=5, temperature=0.0, stop_strings=["\n"])
        assert c.max_tokens == 5 and c.stop_strings == ["\n"]

    def test_gbnf_builders(self):
        assert "json_mode" in repr(GbnfConstraint.json_mode())
        assert "integer" in repr(GbnfConstraint.integer())
        assert "identifier" in repr(GbnfConstraint.identifier())
        assert "choice" in repr(GbnfConstraint.choice(["a", "b"]))
        with pytest.raises(ValueError):
            GbnfConstraint.choice([])
        with pytest.raises(ValueError):
            GbnfConstraint.from_grammar("root ::= (")
        assert GbnfConstraint.from_grammar('root ::= "x"')

    def test_exports(self):
        for n in ("astream", "TokenChannel", "load", "shutdown_stream_executor", "Engine", "Metrics"):
            assert n in air_rs.__all__
        assert inspect.isasyncgenfunction(air_rs.astream)
        air_rs.shutdown_stream_executor()
        air_rs.shutdown_stream_executor()
        ex = air_rs._get_executor()
        assert ex is air_rs._get_executor()
        air_rs.shutdown_stream_executor()


@pytest.fixture(scope="module")
def engine(tmp_path_factory):
    p = tmp_path_factory.mktemp("m") / "tiny.gguf"
    write_random_gguf(str(p), tiny_llama(), GGMLType.Q8_0, seed=0)
    return air_rs.Engine.from_gguf(str(p), device="cpu", temperature=0.0)


class TestEngineCPU:
    def test_generate_returns_string(self, engine):
        out = engine.generate("hello", GenerateConfig(max_tokens=8, temperature=0.0))
        assert isinstance(out, str)
        m = engine.metrics()
        assert m.generated_tokens >= 1 and m.prompt_tokens == 6 and m.total_time_ms > 0

    def test_greedy_is_deterministic_and_reset(self, engine):
        a = engine.generate("abc", GenerateConfig(max_tokens=6, temperature=0.0))
        engine.reset()
        b = engine.generate("abc", GenerateConfig(max_tokens=6, temperature=0.0))
        assert a == b

    def test_stream_to_list_matches_generate(self, engine):
        cfg = GenerateConfig(max_tokens=6, temperature=0.0)
        assert "".join(engine.stream_to_list("xyz", cfg)) == engine.generate("xyz", cfg)

    def test_grammar_choice_constrains_output(self, engine):
        engine.set_grammar(GbnfConstraint.choice(["A", "BB"]))
        assert engine.has_grammar()
        out = engine.generate("q", GenerateConfig(max_tokens=5, temperature=0.0))
        engine.clear_grammar()
        assert out in ("A", "BB")
        assert not engine.has_grammar()

    def test_stop_strings(self, engine):
        toks = engine.stream_to_list("s", GenerateConfig(max_tokens=12, temperature=0.0))
        assert len(toks) >= 3
        # a stop string is matched against the end of the generated text and removed
        cut = engine.generate("s", GenerateConfig(max_tokens=12, temperature=0.0, stop_strings=[toks[2]]))
        assert cut == "".join(toks[:2]) or toks[2] in "".join(toks[:2])

    def test_astream_yields_strings_and_loop_alive(self, engine):
        async def run():
            ticks = 0

            async def ticker():
                nonlocal ticks
                while True:
                    ticks += 1
                    await asyncio.sleep(0.001)

            t = asyncio.ensure_future(ticker())
            toks = [tok async for tok in air_rs.astream(engine, "hi", GenerateConfig(max_tokens=5, temperature=0.0))]
            t.cancel()
            return toks, ticks
        toks, ticks = asyncio.run(run())
        assert all(isinstance(t, str) for t in toks) and len(toks) >= 1
        assert ticks > 0
