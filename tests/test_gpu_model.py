"""The whole decode path (28 layers, vocab head, argmax, generate loop)
through the C ABI vs the CPU oracle, for each engine against the oracle in
that engine's summation orders: logits bit for bit, greedy tokens
identical over 256 steps, the reference's end-of-text
rule, and the chat state machine."""
import numpy as np
import pytest
from conftest import bits

pytestmark = pytest.mark.gpu

EOS = 151645


@pytest.fixture(params=["persistent", "graph", "fused"])
def engine(request):
    return request.param


@pytest.fixture(scope="module")
def oracles(gpu, O, model_weights):
    from q3b200.weights import to_oracle_dict

    dw = gpu.DeviceWeights(model_weights)
    od = to_oracle_dict(model_weights)
    return dw, {"exact": O.Model(od, order=O.ORDER_EXACT), "fused": O.Model(od, order=O.ORDER_FUSED)}


@pytest.fixture
def models(oracles, engine):
    """(device weights, the oracle in the engine's summation orders)"""
    dw, oms = oracles
    return dw, oms["fused" if engine == "fused" else "exact"]


def test_decode_steps_bit_exact(gpu, O, models, engine):
    dw, om = models
    S = 64
    dec = gpu.Qwen3Decoder(dw, max_seq_len=S, engine=engine)
    kc, vc = om.new_cache(S)
    tok = 9
    for pos in range(4):
        logits, nxt = dec.decode(tok, pos)
        otok, ologits = om.decode_step(tok, pos, kc, vc, S)
        assert np.array_equal(bits(logits), bits(ologits)), pos
        assert nxt == otok
        tok = nxt
    dec.close()


def test_run_256_greedy_tokens_identical(gpu, O, models, engine):
    """32 prompt ids U[0,151936), 256 generated, cache 1024."""
    dw, om = models
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, 151936, size=32, dtype=np.int64)
    dec = gpu.Qwen3Decoder(dw, max_seq_len=1024, engine=engine)
    out, n = dec.run(prompt, 256, EOS)
    assert dec.device_error() == 0
    want, _, _ = om.generate(prompt, 256, EOS, 1024)
    assert n == len(want)
    mism = np.nonzero(out[:n] != want)[0]
    assert mism.size == 0, f"first mismatch at step {mism[:1]}"
    dec.close()


def test_eos_rule_matches_reference(gpu, O, models, engine):
    """@generate stops only when the LAST token of a group of 4 is eos
    (model/qwen3_full.mlir:1412-1419, :1528-1530)."""
    dw, om = models
    prompt = np.array([1, 2, 3], np.int64)
    dec = gpu.Qwen3Decoder(dw, max_seq_len=64, engine=engine)
    free, n = dec.run(prompt, 12, -7)
    assert n == 12
    # eos equal to the last token of the first group: stops after 4 tokens
    out, n2 = dec.run(prompt, 12, int(free[3]))
    assert n2 == 4 and np.array_equal(out[:4], free[:4])
    # eos seen mid-group does not stop the loop
    eos = int(free[1])
    expect = next((g for g in (4, 8, 12) if free[g - 1] == eos), 12)
    out, n3 = dec.run(prompt, 12, eos)
    want, _, _ = om.generate(prompt, 12, eos, 64)
    assert n3 == expect == len(want) and np.array_equal(out[:n3], want)
    dec.close()


def test_chat_turns_match_oracle(gpu, O, models, engine):
    """@init_chat/@chat_turn: zero cache, turn = ingest + generate, then the
    position moves by n_tokens + n_out + 1 (model/qwen3_full.mlir:2216-2218)."""
    dw, om = models
    S = 128
    dec = gpu.Qwen3Decoder(dw, max_seq_len=S, engine=engine)
    dec.init_chat(S)
    kc, vc = om.new_cache(S)
    pos = 0
    for turn, toks in enumerate([np.array([10, 20, 30], np.int64), np.array([40], np.int64)]):
        out, n = dec.chat_turn(toks, 6, -7)
        assert n == 6
        tok = None
        for i, t in enumerate(toks):
            tok, _ = om.decode_step(int(t), pos + i, kc, vc, S)
        p = pos + len(toks)
        want = []
        for _ in range(6):
            nxt, _ = om.decode_step(tok, p, kc, vc, S)
            want.append(nxt)
            tok, p = nxt, p + 1
        assert np.array_equal(out[:n], want), turn
        pos = pos + len(toks) + n + 1
    dec.close()
