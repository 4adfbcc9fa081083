"""Failure detection without a GPU fault.

* A bounded device wait on a flag that nothing sets runs out after its short
  limit, records its code in the error word, the host call reports
  Q3_ERR_DEVICE, and the context stays usable (the next kernels run and are
  exact).
* A corrupted decode state -- an out-of-range token or position written on
  the host through the test hook q3_model_poke -- reaches the kernels' checks
  (kErrBadToken = 4, kErrBadPos = 5) on every engine; nothing outside the
  buffers is touched, the call returns Q3_ERR_DEVICE, and a new generation on
  the same model is exact again."""
import ctypes

import numpy as np
import pytest
from conftest import bits

pytestmark = pytest.mark.gpu

ERR_WAIT, ERR_TOKEN, ERR_POS = 3, 4, 5


def test_bounded_wait_expires_and_reports(gpu, O):
    L = gpu.lib()
    flag = gpu.DeviceArray((1,), np.int32, zero=True)
    err = gpu.DeviceArray((1,), np.int32, zero=True)
    # nothing ever sets the flag: the wait gives up after ~1 ms of SM clock
    assert L.q3_selftest_bounded_wait(flag.ptr, 1, 2_000_000, err.ptr, None) == 0
    assert L.q3_check_error_word(err.ptr, None) == 3  # Q3_ERR_DEVICE
    assert b"error word 3" in L.q3_last_error()
    assert int(err.download()[0]) == ERR_WAIT
    # a flag that is set ends the wait without an error
    flag.upload(np.array([1], np.int32))
    err.zero()
    assert L.q3_selftest_bounded_wait(flag.ptr, 1, 2_000_000, err.ptr, None) == 0
    assert L.q3_check_error_word(err.ptr, None) == 0
    # the context is intact: a GEMV afterwards is still exact
    rng = np.random.default_rng(3)
    w = O.quantize_q8_0_c((rng.standard_normal((256, 1024)) * 0.02).astype(np.float32))
    x = rng.standard_normal(1024).astype(np.float16)
    dw, dx, dy = gpu.DeviceArray.from_host(w), gpu.DeviceArray.from_host(x), gpu.DeviceArray((256,), np.float16)
    assert L.q3_gemv_q8(dw.ptr, dx.ptr, dy.ptr, 256, 1024, None) == 0
    assert np.array_equal(bits(dy.download()), bits(O.gemv_q8(w, x, 256, 1024)))


def test_bounded_wait_rejects_limits_above_the_budget(gpu):
    L = gpu.lib()
    buf = gpu.DeviceArray((2,), np.int32, zero=True)
    assert L.q3_selftest_bounded_wait(buf.ptr, 1, 10**12, buf.ptr + 4, None) == 1


@pytest.fixture(scope="module")
def fmodels(gpu, O, model_weights):
    from q3b200.weights import to_oracle_dict

    od = to_oracle_dict(model_weights)
    return gpu.DeviceWeights(model_weights), {
        "graph": O.Model(od, order=O.ORDER_EXACT), "fused": O.Model(od, order=O.ORDER_FUSED)}


@pytest.mark.parametrize("engine", ["graph", "fused"])
@pytest.mark.parametrize("what,value,code", [(0, 10**9, ERR_TOKEN), (0, -3, ERR_TOKEN),
                                             (1, 10**6, ERR_POS), (1, -1, ERR_POS)])
def test_corrupted_state_is_reported_not_faulted(gpu, fmodels, engine, what, value, code):
    from q3b200._lib import Q3Error

    dw, oms = fmodels
    S = 64
    dec = gpu.Qwen3Decoder(dw, max_seq_len=S, engine=engine)
    prompt = np.array([5, 6, 7], np.int64)
    dec.generate_begin(prompt, 6, -1)
    # the next step reads the token at position 3 (its input) and position 3 itself
    idx = 3
    assert gpu.lib().q3_model_poke(dec.handle, what, idx, value) == 0
    dec.generate_steps(2)
    with pytest.raises(Q3Error) as e:
        dec.generate_end(6)
    assert e.value.status == 3  # Q3_ERR_DEVICE
    assert dec.device_error() == code
    # the same model decodes exactly again
    out, n = dec.run(prompt, 6, -1)
    want, _, _ = oms["fused" if engine == "fused" else "graph"].generate(prompt, 6, -1, S)
    assert dec.device_error() == 0 and n == 6 and np.array_equal(out[:n], want)
    dec.close()
