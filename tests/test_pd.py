"""Prefill/decode disaggregation: wire format, connectors with timeouts / corruption /
back-pressure (host fault injection), and the device KV push between two engines."""
import struct

import pytest
import torch

from air_rs.parallel.pd import (DecodeNode, KvBlock, KvTransferError, PdDisaggConfig, PrefillNode, ShmKvConnector,
                                TcpKvConnector, blocks_from_pool, decode_frame, encode_frame)


def test_kvblock_wire_format_matches_reference_layout():
    b = KvBlock(7, 3, b"\x01\x02\x03")
    s = b.serialise()
    assert s[:10] == struct.pack("<IHI", 7, 3, 3) and s[10:] == b"\x01\x02\x03"
    assert KvBlock.deserialise(s) == b and KvBlock.deserialise(s[:9]) is None
    q, sc = KvBlock.int8_quantize(torch.tensor([0.5, -1.0, 0.25]).bfloat16())
    assert q.tolist() == [64, -127, 32] and abs(sc - 1 / 127) < 1e-9


def test_frame_checksum_detects_corruption():
    f = bytearray(encode_frame(5, [KvBlock(1, 0, b"abcd"), KvBlock(2, 1, b"efgh")]))
    assert decode_frame(bytes(f))[0] == 5
    f[-6] ^= 0x10
    with pytest.raises(KvTransferError) as e:
        decode_frame(bytes(f))
    assert e.value.kind == "corrupt"


def _pool(seed=0):
    return torch.randn(2, 8, 2, 2, 4, 8, generator=torch.Generator().manual_seed(seed)).bfloat16()


@pytest.mark.parametrize("quantize", [True, False])
def test_shm_prefill_to_decode_roundtrip(quantize):
    cfg = PdDisaggConfig(transfer_timeout=0.5)
    conn = ShmKvConnector()
    src, dst = _pool(0), torch.zeros(2, 8, 2, 2, 4, 8).bfloat16()
    n = PrefillNode(cfg, conn).prefill_and_send(11, src, [1, 4], quantize)
    assert n == 4
    DecodeNode(cfg, conn).recv_and_prepare(11, dst, {1: 6, 4: 0}, n_layers=2, quantize=quantize)
    tol = 0.02 if quantize else 0.0
    torch.testing.assert_close(dst[:, 6].float(), src[:, 1].float(), rtol=0, atol=tol * 4)
    torch.testing.assert_close(dst[:, 0].float(), src[:, 4].float(), rtol=0, atol=tol * 4)


def test_dropped_frame_times_out_and_is_counted():
    cfg = PdDisaggConfig(transfer_timeout=0.2)
    conn = ShmKvConnector()
    conn.drop_next = True
    PrefillNode(cfg, conn).prefill_and_send(3, _pool(), [0])
    dec = DecodeNode(cfg, conn)
    with pytest.raises(KvTransferError) as e:
        dec.recv_and_prepare(3, torch.zeros(2, 8, 2, 2, 4, 8).bfloat16(), {0: 0}, n_layers=2)
    assert e.value.kind == "timeout" and dec.metrics.timeouts_total == 1


def test_backpressure_refuses_beyond_max_in_flight():
    cfg = PdDisaggConfig(max_in_flight=0)
    with pytest.raises(KvTransferError) as e:
        PrefillNode(cfg, ShmKvConnector()).prefill_and_send(1, _pool(), [0])
    assert e.value.kind == "partial"


def test_tcp_connector_roundtrip_and_corruption():
    rx = TcpKvConnector()
    port = rx.listen()
    tx = TcpKvConnector()
    blocks = blocks_from_pool(_pool(2), [3], quantize=False)
    tx.send_blocks(9, blocks, ("127.0.0.1", port))
    got = rx.recv_blocks(9, len(blocks), timeout=5.0)
    assert [b.data for b in got] == [b.data for b in blocks]
    tx.send_blocks(10, blocks, ("127.0.0.1", port), corrupt=True)
    with pytest.raises(KvTransferError) as e:
        rx.recv_blocks(10, len(blocks), timeout=5.0)
    assert e.value.kind == "corrupt"
    with pytest.raises(KvTransferError) as e:
        rx.recv_blocks(11, 1, timeout=0.1)
    assert e.value.kind == "timeout"
    rx.close()


@pytest.mark.gpu
def test_device_kv_push_handoff_matches_single_engine():
    from air_rs.gguf import GGMLType
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import random_tensors
    from air_rs.models.reference import OracleModel
    from air_rs.parallel.pd import PdPair
    from air_rs.runtime.builder import build_runner
    from air_rs.runtime.engine import Engine, SamplingParams
    from test_engine_gpu import _check_near_argmax
    cfg = tiny_llama()
    recs = list(random_tensors(cfg, GGMLType.Q8_0, seed=0, device="cpu"))
    oracle = OracleModel(cfg, {n: (r, q, s) for n, r, q, s in recs})
    dev_d = "cuda:1" if torch.cuda.device_count() > 1 else "cuda:0"
    pre = Engine(cfg, build_runner(cfg, iter(recs), device="cuda:0", max_batch=8, max_model_len=256, num_blocks=64))
    dec = Engine(cfg, build_runner(cfg, iter(recs), device=dev_d, max_batch=8, max_model_len=256, num_blocks=64))
    pair = PdPair(pre, dec)
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, cfg.vocab_size, (int(n),), generator=g).tolist() for n in (37, 12)]
    sp = SamplingParams(max_tokens=16, temperature=0.0, repetition_penalty=1.0, ignore_eos=True)
    rids = [pair.submit(p, sp, verify=True) for p in prompts]
    with torch.cuda.device(dec.runner.device):
        while dec.has_unfinished():
            dec.step()
    for rid, p in zip(rids, prompts):
        out = dec.finished[rid].output_ids
        assert len(out) == 16
        _check_near_argmax(oracle, [cfg.bos_token_id] + p, out, penalty=1.0)
    assert pair.metrics.transfers_total == 2 and pre.seqs.allocator.num_used_blocks() == 0


def test_warp_header_and_handshake_codec():
    from air_rs.parallel.pd import (FEAT_INT8, FEAT_LZ4, WARP_HEADER, decode_handshake, encode_handshake,
                                    parse_warp_header, warp_header)
    h = warp_header(FEAT_INT8, 1234)
    assert len(h) == WARP_HEADER.size == 18 and h[:4] == b"WARP"
    assert parse_warp_header(h) == (FEAT_INT8, 1234)
    for bad, why in [(b"XARP" + h[4:], "magic"), (h[:4] + (0x0201).to_bytes(2, "little") + h[6:], "major"),
                     (warp_header(FEAT_LZ4, 5), "unsupported")]:
        with pytest.raises(KvTransferError, match=why) as e:
            parse_warp_header(bad)
        assert e.value.kind == "protocol"
    assert parse_warp_header(h[:4] + (0x0107).to_bytes(2, "little") + h[6:])[1] == 1234   # minor differs: ok
    body = encode_handshake(b"\x01" * 32, "llama-3-8b")
    assert decode_handshake(body) == (b"\x01" * 32, "llama-3-8b")
    with pytest.raises(KvTransferError):
        decode_handshake(body[:-1])


def test_tcp_connector_rejects_another_models_stream(tmp_path):
    from air_rs.gguf import GGMLType
    from air_rs.models.config import tiny_llama
    from air_rs.models.random_init import write_random_gguf
    from air_rs.parallel.pd import FEAT_INT8, gguf_fingerprint
    a, b = tmp_path / "a.gguf", tmp_path / "b.gguf"
    write_random_gguf(str(a), tiny_llama(), GGMLType.Q8_0, seed=0)
    write_random_gguf(str(b), tiny_llama(), GGMLType.Q4_K, seed=0)
    fa, fb = gguf_fingerprint(str(a)), gguf_fingerprint(str(b))
    assert len(fa) == 32 and fa == gguf_fingerprint(str(a)) and fa != fb
    rx = TcpKvConnector(fingerprint=fa, model_name="a")
    port = rx.listen()
    blocks = blocks_from_pool(_pool(2), [1], quantize=True)
    TcpKvConnector(fingerprint=fa, model_name="a").send_blocks(1, blocks, ("127.0.0.1", port), features=FEAT_INT8)
    assert len(rx.recv_blocks(1, len(blocks), timeout=5.0)) == len(blocks)
    assert rx.peers == [(fa, "a")]
    TcpKvConnector(fingerprint=fb, model_name="b").send_blocks(2, blocks, ("127.0.0.1", port))
    with pytest.raises(KvTransferError) as e:
        rx.recv_blocks(2, len(blocks), timeout=5.0)
    assert e.value.kind == "handshake" and "'b'" in str(e.value)
    rx.close()
