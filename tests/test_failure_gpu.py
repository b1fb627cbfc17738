"""GPU failure detection without a GPU fault.

The TMA-staged GEMV waits on shared-memory copies through mbarriers; every
wait is bounded (about a second).  The test hook withholds the copies of one
row tile so its wait can never complete: the kernel must give up, set the
device error flag, let its other copies land and exit, leaving the context
usable.  Nothing here faults, traps or hangs the GPU.
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_context_survives(pkg, orc, S, cuda):
    torch = cuda
    L = pkg.lib()
    assert L.dqmk_device_error(1) == 0  # clean start
    blocks, x = S.gemv_case(64, 896, 3)
    packed = pkg.pack_weight(pkg.Q80, blocks, 64, 896)
    xd = torch.from_numpy(x).cuda()
    y = torch.zeros(64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.time()
    pkg.check(L.dqmk_gemv_packed_withhold_tile(pkg.Q80, xd.data_ptr(), 896, packed.data_ptr(),
                                               64, y.data_ptr(), 2, stream))
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert waited < 30, waited
    assert L.dqmk_device_error(1) & 1  # the timeout was recorded ...
    assert L.dqmk_device_error(0) == 0  # ... and cleared by the read
    # the context still works: the same GEMV, nothing withheld, matches the oracle
    y2 = pkg.gemv_packed(pkg.Q80, xd, packed, 64).cpu().numpy()
    ref = orc.linear(pkg.Q80, x, blocks, 64)
    assert np.abs(y2 - ref).max() <= 1e-3 * max(1.0, np.abs(ref).max())
    assert L.dqmk_device_error(0) == 0


def test_lm_head_timeout_keeps_greedy_state(pkg, orc, S, cuda):
    """Every row tile of the decode step's lm_head withheld for two greedy
    steps: each CTA's bounded wait runs out, no row is scored, so no token id
    exists for the step.  The greedy state (token, position, history) must be
    kept -- never an invalid id fed to the next step's embedding -- and the call
    must report the timeout.  With the hook removed, the same context decodes
    the reference context's greedy tokens from the same token and position.
    The model is Qwen2-shaped with a 40960-id vocabulary so its tied lm_head is
    the TMA-staged (bounded-wait) GEMV."""
    L = pkg.lib()
    assert L.dqmk_device_error(1) == 0
    cfg = dict(S.QWEN2_MINI, vocab=40960, n_layers=1)
    w = S.make_model(cfg, S.Q80, 21, quantize_q80=orc.quantize_q80)
    model = pkg.Model.from_synth(w, max_seq_len=16)
    ref = pkg.Context(model)
    tok = int(np.argmax(ref.ForwardToken(5, 0)))
    ref_tokens = ref.decode_greedy(tok, 1, 4).tolist()
    ref.close()

    ctx = pkg.Context(model)
    ctx.ForwardToken(5, 0)
    pkg.check(L.dqmk_context_withhold_lm_head(ctx.h, -2))
    t0 = time.time()
    with pytest.raises(pkg.CudaError, match="no scored token"):
        ctx.decode_greedy(tok, 1, 2)
    assert time.time() - t0 < 60
    assert L.dqmk_device_error(0) == 0  # the call read and cleared the flags
    pkg.check(L.dqmk_context_withhold_lm_head(ctx.h, -1))
    assert ctx.decode_greedy(tok, 1, 4).tolist() == ref_tokens
    assert L.dqmk_device_error(0) == 0
    ctx.close()
    model.close()
