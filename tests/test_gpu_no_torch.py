"""The forward on the GPU in a process that never imports torch: the layer pipeline, the native
network plan, the pipelined host-in/host-out forward and the float layer, checked against the
oracle (bit for bit / within the float tolerance); torch must still be absent at the end."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

_SCRIPT = """
import sys
sys.path[:0] = [{root!r}, {root!r} + '/oracle', {root!r} + '/tests']
import numpy as np
import oracle as O
import salt_b200 as S
from salt_b200 import device as D
from salt_b200.plan import NetworkPlan, PipelinedForward
from _cases import make_events, make_params
rng = np.random.default_rng(5)
net = S.Network.build((2, 12, 12), [
    S.conv(16, k=3, s=2, p=0, init_k=5.0, tau=20.0, max_queue_len=64, max_out_spikes=600),
    S.conv(32, k=3, s=2, p=1, init_k=5.0, tau=20.0, max_queue_len=64, max_out_spikes=400),
    S.fc(10, init_k=5.0, tau=20.0, v_th=1e9, max_out_spikes=1)])
params = [make_params(l, rng, vth=(60, 160), fires=i < 2) for i, l in enumerate(net.layers)]
B, E = 8, 300
times, src, nr = make_events(rng, B, E, 2 * 12 * 12)
out = net.apply_batched(params, S.InputEvents.checked(times, src, nr), keep_streams=True)
ref = [O.network_forward(net.layers, params, times[b], src[b], nr[b]) for b in range(B)]
for b in range(B):
    assert np.array_equal(out.last.v_final[b], ref[b][-1].v_final)
    assert np.array_equal(out.streams[0].event_source_idx[b], ref[b][0].event_source_idx)
plan = NetworkPlan(net.layers, params, B, E)
logits, stats, fits = plan(S.InputEvents(times, src, nr))
assert np.array_equal(logits, out.last.v_final)
pf = PipelinedForward(net.layers, params, B, E, chunks=2)
lg, ft = pf(D.pinned_copy(times), D.pinned_copy(src), D.pinned_copy(nr, np.int32))
assert np.array_equal(lg, logits) and np.array_equal(ft != 0, fits)
pf.close()
fl = S.FCLayer(name='f', n_in=2 * 12 * 12, n_out=24, init_k=1.0, tau=16.0, v_th=1.0,
               chunk_size=8, max_out_spikes=4000, max_extra_steps=300)
w = rng.normal(0.0, 0.3, (24, 2 * 12 * 12)).astype(np.float32)
fo = S.FloatB200Backend().forward_layer(fl, w, S.EventStream(times, src, np.ones_like(times), nr))
for b in range(B):
    r = O.float_fc_forward(fl, w, times[b], src[b], int(nr[b]), dense=False)
    assert np.allclose(fo.result.v_final[b], r.v_final, rtol=1e-5, atol=1e-6)
assert 'torch' not in sys.modules
print('ok')
"""


def test_forward_without_torch_in_the_process():
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _SCRIPT.format(root=root)], capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), (r.stdout[-1000:],
                                                                   r.stderr[-3000:])
