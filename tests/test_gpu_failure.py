"""In-kernel bounded waits on the GPU: a wait that runs out ends in an error status
the host reads, and the context stays usable (the contract that device work ends
before any rollback, miniprefix/include/miniprefix/kv_manager.h:36-38).

mp_inject_wait_timeout makes the next forward's first GEMM launch issue no copies
with its waits bounded at 1 ms, so the MMA issuer's and the epilogue's mbarrier
waits expire (a barrier nothing completes). The kernel records the timeout bit,
releases its tensor memory and returns; the forward reports MP_ERR_TIMEOUT within
milliseconds rather than the default 2 s bound. The next forwards on the same
context -- in another slot, then over the slot the failed step wrote garbage
into -- match the C oracle."""
import time

import numpy as np
import pytest

from oracle.oracle import Oracle
from tinyinfer_b200.synthetic import ModelConfig, random_tokens, random_weights


@pytest.mark.gpu
def test_expired_in_kernel_wait_reports_timeout_and_context_recovers(built):
    from tinyinfer_b200.device import MP_ERR_TIMEOUT, DeviceContext, DeviceError

    cfg = ModelConfig(layers=2, context=64)
    w = random_weights(cfg, seed=8)
    o = Oracle(cfg, w, 16)
    ctx = DeviceContext(cfg, device=0, block_tokens=16, max_blocks=8, max_sequences=2, max_step_tokens=16,
                        max_step_sequences=2)
    ctx.load_weights(w)
    ctx.table_write(0, 0, [0])
    ctx.table_write(1, 0, [1])
    prompt = random_tokens(9, cfg.vocabulary, 3)
    keys, values = o.new_pools(2)
    expect, _ = o.append(keys, values, [0], 0, prompt)

    ctx.inject_wait_timeout(1000)
    t0 = time.perf_counter()
    with pytest.raises(DeviceError) as e:
        ctx.forward([(0, 0, 9)], prompt)
    assert e.value.code == MP_ERR_TIMEOUT
    assert time.perf_counter() - t0 < 1.5  # the 1 ms bound, not the default 2 s

    for slot in (1, 0):
        t, f, logits, rc = ctx.forward([(slot, 0, 9)], prompt)
        assert rc == 0 and f.all()
        assert (np.abs(logits[0] - expect) <= 1e-3 + 1e-4 * np.abs(expect)).all()
        assert int(t[0]) == int(np.argmax(expect))
    ctx.close()
