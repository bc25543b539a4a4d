"""The pipelined host-in/host-out forward (sub-batches with overlapped transfers that move only
each sample's real events) equals the plain batched plan, including a first layer that fires on
pad entries (whole rows are then copied) and samples without events."""
import ctypes

import numpy as np
import pytest

import salt_b200 as S
from salt_b200 import device as D
from salt_b200.plan import NetworkPlan, PipelinedForward
from _cases import make_events, make_params

pytestmark = pytest.mark.gpu


def _net(rng, vth):
    net = S.Network.build((2, 12, 12), [
        S.conv(8, k=3, s=2, p=0, init_k=5.0, tau=20.0, max_queue_len=96, max_out_spikes=900),
        S.conv(16, k=3, s=2, p=1, init_k=5.0, tau=20.0, max_queue_len=96, max_out_spikes=600),
        S.fc(7, init_k=5.0, tau=20.0, v_th=1e9, max_out_spikes=1)])
    params = [make_params(l, rng, vth=vth, fires=i < 2) for i, l in enumerate(net.layers)]
    return net, params


@pytest.mark.parametrize("vth,chunks", [((60, 160), 4), ((60, 160), 2), ((-10, 30), 4)])
def test_pipelined_equals_the_batched_plan(vth, chunks):
    rng = np.random.default_rng(9)
    net, params = _net(rng, vth)
    B, E = 24, 400
    times, src, nr = make_events(rng, B, E, 2 * 12 * 12, pad_time="big")
    nr[3], nr[7] = 0, E + 50
    plan = NetworkPlan(net.layers, params, B, E)
    ref_logits, _, ref_fits = plan.forward_device(D.to_device(times, np.float32),
                                                  D.to_device(src, np.int32),
                                                  D.to_device(nr, np.int32))
    ref_logits, ref_fits = ref_logits.numpy(), ref_fits.numpy()
    pf = PipelinedForward(net.layers, params, B, E, chunks=chunks)
    assert pf.full_rows == (vth[0] <= 0)
    t_h, s_h, n_h = D.pinned_copy(times), D.pinned_copy(src), D.pinned_copy(nr, np.int32)
    for _ in range(2):   # twice: the second call starts from the first call's buffers
        logits, fits = pf(t_h, s_h, n_h)
        np.testing.assert_array_equal(logits, ref_logits)
        np.testing.assert_array_equal(fits, ref_fits)
    assert pf.h2d_bytes(nr) <= B * E * 8 + B * 4
    pf.close()


def test_back_to_back_calls_without_host_sync():
    """Calls enqueued back to back (sync=False): a call's first sub-batches reuse the device
    buffers that the previous call's last sub-batches still read."""
    rng = np.random.default_rng(11)
    net, params = _net(rng, (60, 160))
    B, E = 32, 600
    sets = []
    for _ in range(3):
        times, src, nr = make_events(rng, B, E, 2 * 12 * 12)
        sets.append((D.pinned_copy(times), D.pinned_copy(src), D.pinned_copy(nr, np.int32)))
    plan = NetworkPlan(net.layers, params, B, E)
    refs = [plan.forward_device(D.to_device(t, np.float32), D.to_device(s, np.int32),
                                D.to_device(n, np.int32))[0].numpy() for t, s, n in sets]
    pf = PipelinedForward(net.layers, params, B, E, chunks=4)
    out = D.empty((6, B, pf.plan.n_out), np.int32)
    for r in range(6):
        pf(*sets[r % 3], sync=False)
        out[r].copy_from_device(pf.plan.logits)   # stream-ordered after the call's forward
    got = out.numpy()
    for r in range(6):
        np.testing.assert_array_equal(got[r], refs[r % 3])
    pf.close()


def test_unpinned_host_rows_are_rejected():
    from salt_b200 import _lib
    t = np.zeros((2, 8), np.float32)          # pageable
    s = np.zeros((2, 8), np.int32)
    n = D.zeros((2,), np.int32)
    dt = D.empty((2, 8), np.float32)
    ds = D.empty((2, 8), np.int32)
    rc = _lib.lib().salt_stream_h2d_real(D.ptr(t), D.ptr(s), ctypes.c_int64(8), D.ptr(n), 2, 8,
                                         D.ptr(dt), D.ptr(ds), None)
    assert rc == _lib.SALT_BAD_ARG


def test_forward_parts_in_any_slicing_equal_the_full_forward():
    """salt_network_forward_part: layer 0 on uneven row slices, layer 1 on two slices, the last
    layer on all rows gives the full forward's logits, fits and per-layer stats."""
    rng = np.random.default_rng(13)
    net, params = _net(rng, (60, 160))
    B, E = 10, 300
    times, src, nr = make_events(rng, B, E, 2 * 12 * 12)
    t, s, n = D.to_device(times, np.float32), D.to_device(src, np.int32), D.to_device(nr, np.int32)
    full = NetworkPlan(net.layers, params, B, E)
    lf, sf, ff = (x.numpy() for x in full.forward_device(t, s, n))
    part = NetworkPlan(net.layers, params, B, E)
    for r0, r1 in ((0, 3), (3, 4), (4, 10)):
        part.forward_part(t[r0:r1], s[r0:r1], n[r0:r1], r0, r1 - r0, 0, 1)
    for r0, r1 in ((0, 6), (6, 10)):
        part.forward_part(None, None, None, r0, r1 - r0, 1, 2)
    lp, sp, fp = part.forward_part(None, None, None, 0, B, 2, 3)
    np.testing.assert_array_equal(lp.numpy(), lf)
    np.testing.assert_array_equal(fp.numpy(), ff)
    np.testing.assert_array_equal(sp.numpy(), sf)


def test_captured_graph_replays_the_forward():
    """NetworkPlan.capture: a CUDA graph of the forward gives the eager results, and replays
    pick up new contents of the captured input buffers."""
    rng = np.random.default_rng(17)
    net, params = _net(rng, (60, 160))
    B, E = 12, 300
    plan = NetworkPlan(net.layers, params, B, E)
    t, s, n = D.empty((B, E), np.float32), D.empty((B, E), np.int32), D.empty((B,), np.int32)
    sets = [make_events(rng, B, E, 2 * 12 * 12) for _ in range(2)]
    t.copy_from(sets[0][0], sync=True)
    s.copy_from(sets[0][1], sync=True)
    n.copy_from(sets[0][2].astype(np.int32), sync=True)
    replay = plan.capture(t, s, n)
    eager = NetworkPlan(net.layers, params, B, E)
    for times, src, nr in sets:
        t.copy_from(times, sync=True)
        s.copy_from(src, sync=True)
        n.copy_from(nr.astype(np.int32), sync=True)
        replay()
        lg, st, ft = eager.forward_device(t, s, n)
        np.testing.assert_array_equal(plan.logits.numpy(), lg.numpy())
        np.testing.assert_array_equal(plan.stats.numpy(), st.numpy())
        np.testing.assert_array_equal(plan.fits.numpy(), ft.numpy())


def test_network_whose_last_layer_fires():
    """A firing last layer compacts its full output stream inside the network workspace (the
    single firing FC layer of configuration 1; a conv net ending in a firing conv)."""
    import oracle as O
    rng = np.random.default_rng(19)
    for net in (S.Network.build((2, 12, 12), [
                    S.fc(128, init_k=5.0, tau=20.0, max_out_spikes=700)]),
                S.Network.build((2, 12, 12), [
                    S.conv(8, k=3, s=2, p=0, init_k=5.0, tau=20.0, max_queue_len=96,
                           max_out_spikes=900),
                    S.conv(16, k=3, s=2, p=1, init_k=5.0, tau=20.0, max_queue_len=96,
                           max_out_spikes=500)])):
        params = [make_params(l, rng, vth=(60, 160)) for l in net.layers]
        B, E = 3, 400
        times, src, nr = make_events(rng, B, E, 2 * 12 * 12)
        plan = NetworkPlan(net.layers, params, B, E)
        logits, stats, fits = plan.forward_device(D.to_device(times, np.float32),
                                                  D.to_device(src, np.int32),
                                                  D.to_device(nr, np.int32))
        logits, stats = logits.numpy(), stats.numpy()
        for b in range(B):
            refs = O.network_forward(net.layers, params, times[b], src[b], nr[b])
            np.testing.assert_array_equal(logits[b], refs[-1].v_final)
            assert [int(v) for v in stats[0, :, b]] == [r.n_real_events for r in refs]


def test_overlapped_batches_equal_the_batched_plan():
    """Two batches in flight (two plans on two streams): every submission's logits, stats and
    fits equal a single plan's forward of the same batch, with the outputs read on a stream that
    waits only for that submission's done event, and a held event delaying a plan's reuse."""
    from salt_b200.plan import OverlappedForward
    rng = np.random.default_rng(13)
    net, params = _net(rng, (60, 160))
    B, E = 32, 600
    sets = []
    for _ in range(3):
        times, src, nr = make_events(rng, B, E, 2 * 12 * 12)
        sets.append((D.to_device(times, np.float32), D.to_device(src, np.int32),
                     D.to_device(nr, np.int32)))
    plan = NetworkPlan(net.layers, params, B, E)
    refs = []
    for t, s, n in sets:
        logits, stats, fits = plan.forward_device(t, s, n)
        refs.append((logits.numpy(), stats.numpy(), fits.numpy()))
    ov = OverlappedForward(net.layers, params, B, E)
    reader = D.Stream()
    out_l = D.empty((7, B, plan.n_out), np.int32)
    out_s = D.empty((7,) + tuple(plan.stats.shape), np.int32)
    out_f = D.empty((7, B), np.int32)
    for r in range(7):
        logits, stats, fits, done = ov.submit(*sets[r % 3])
        reader.wait_event(done)
        out_l[r].copy_from_device(logits, stream=reader)
        out_s[r].copy_from_device(stats, stream=reader)
        out_f[r].copy_from_device(fits, stream=reader)
        ov.hold(D.Event().record(reader))
    ov.join()
    D.synchronize()
    assert ov.last_launch_count() > 0
    for r in range(7):
        ref = refs[r % 3]
        np.testing.assert_array_equal(out_l[r].numpy(), ref[0])
        np.testing.assert_array_equal(out_s[r].numpy(), ref[1])
        np.testing.assert_array_equal(out_f[r].numpy(), ref[2])
    ov.close()
    plan.close()


@pytest.mark.parametrize("chunks", [1, 4])
def test_overlapped_pipelined_calls(chunks):
    """overlap=True: calls enqueued back to back on two plans, each into its own pinned result
    slot, with a device reader of each call's logits holding that plan; all equal the batched
    plan."""
    rng = np.random.default_rng(17)
    net, params = _net(rng, (60, 160))
    B, E = 32, 600
    sets = []
    for _ in range(3):
        times, src, nr = make_events(rng, B, E, 2 * 12 * 12)
        sets.append((D.pinned_copy(times), D.pinned_copy(src), D.pinned_copy(nr, np.int32)))
    plan = NetworkPlan(net.layers, params, B, E)
    refs = []
    for t, s, n in sets:
        logits, _, fits = plan.forward_device(D.to_device(t, np.float32), D.to_device(s, np.int32),
                                              D.to_device(n, np.int32))
        refs.append((logits.numpy(), fits.numpy()))
    pf = PipelinedForward(net.layers, params, B, E, chunks=chunks, overlap=True)
    reader = D.Stream()
    dev = D.empty((7, B, plan.n_out), np.int32)
    slots = [(D.pinned_empty((B, plan.n_out), np.int32), D.pinned_empty((B,), np.int32))
             for _ in range(7)]
    for r in range(7):
        pf(*sets[r % 3], sync=False, out=slots[r])
        reader.wait_event(pf.done)
        dev[r].copy_from_device(pf.plan.logits, stream=reader)
        pf.hold(D.Event().record(reader))
    pf.join()
    D.synchronize()
    got = dev.numpy()
    for r in range(7):
        np.testing.assert_array_equal(slots[r][0], refs[r % 3][0])
        np.testing.assert_array_equal(slots[r][1], refs[r % 3][1])
        np.testing.assert_array_equal(got[r], refs[r % 3][0])
    pf.close()
    plan.close()
