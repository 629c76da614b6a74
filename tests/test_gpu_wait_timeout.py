"""A bounded device wait that runs out: GB_ERR_TIMEOUT, then a clean forward.

The one-launch expert kernel's down work waits for ready flags that the
gate_up tiles publish.  With the test hooks the wait limit drops to 50 ms and
the first gate_up tile's flag is withheld (a flag that nothing sets), so the
down work that needs it gives up: the CTA raises its abort flag, lets its
copies land, frees its tensor memory and returns, and the device status reads
GB_ERR_TIMEOUT.  Nothing faults or hangs.  With the hooks reset, the next
forward must give exactly the output of a forward before the failure.
"""
import time

import numpy as np
import pytest

from gallium_b200 import GalliumError, OssMoEFFN, _lib, synth

pytestmark = pytest.mark.gpu


def test_withheld_ready_flag_times_out_and_the_next_forward_is_clean():
    import torch

    layer = synth.gptoss_layer(n_experts=8, hidden=512, inter=512, seed=13)
    x = torch.from_numpy(synth.tokens(32, 512, seed=3)).cuda()  # 128 positions: one launch
    with OssMoEFFN.load(layer, device=0, max_tokens=32) as moe:
        moe.set_graphs(0)
        good = moe.forward(x).cpu().numpy()
        moe.set_test_hooks(wait_limit_us=50_000, withhold_ready=True)
        t0 = time.time()
        with pytest.raises(GalliumError) as ei:
            moe.forward(x)
        elapsed = time.time() - t0
        assert ei.value.status == _lib.GB_ERR_TIMEOUT
        assert elapsed < 5.0, elapsed
        moe.set_test_hooks(0, False)
        again = moe.forward(x).cpu().numpy()
        assert np.array_equal(again, good)
        again = moe.forward(x).cpu().numpy()
        assert np.array_equal(again, good)
