"""Writes known_answers.json: the hand-computed answers of the reference's own tests and of its
integer-inference spec, transcribed (inputs and expected outputs only) with the file:line each
comes from.  Paths are relative to the reference repository (Salt-Shio/Spiking-Affine-Lazy-
Training).  Run: python tests/golden/make_known_answers.py
"""
import json
import os

CASES = []


def case(kind, source, **kw):
    CASES.append({"kind": kind, "source": source, **kw})


# ---------------------------------------------------------------- fixed point
case("round_shift", "salt_core/tests/test_fixed_point.py:21-26",
     x=[5, -5, 3, -3], shift=1, mode="round", expected=[3, -2, 2, -1])
case("round_shift", "salt_core/tests/test_fixed_point.py:29-33",
     x=[5, 7, -5, -7], shift=2, mode="round", expected=[1, 2, -1, -2])
case("round_shift", "salt_core/tests/test_fixed_point.py:36-40",
     x=[5, -5, 3, -3], shift=1, mode="truncate", expected=[2, -3, 1, -2])
case("round_shift", "salt_core/tests/test_fixed_point.py:43-46",
     x=[3, -3, 0], shift=0, mode="round", expected=[3, -3, 0])
case("round_shift", "salt_core/tests/test_fixed_point.py:43-46",
     x=[3, -3, 0], shift=0, mode="truncate", expected=[3, -3, 0])
case("wide_mul_shift", "salt_core/tests/test_fixed_point.py:72-78",
     a=12, v=40, shift=4, mode="round", expected=30)
case("wide_mul_shift", "salt_core/tests/test_fixed_point.py:81-89",
     a=1, v=-8, shift=4, mode="round", expected=0)
case("wide_mul_shift", "salt_core/tests/test_fixed_point.py:81-89",
     a=1, v=-8, shift=4, mode="truncate", expected=-1)
case("wide_mul_shift", "salt_core/tests/test_fixed_point.py:92-93",
     a=3, v=-7, shift=0, mode="round", expected=-21)
case("wide_mul_shift", "salt_core/tests/test_fixed_point.py:96-98",
     a=0, v=12345, shift=8, mode="round", expected=0)
for mode in ("wrap", "saturate"):
    case("fit_to_bits", "salt_core/tests/test_fixed_point.py:125-130",
         x=[7, -8, 0, 3], total=4, mode=mode, expected=[7, -8, 0, 3],
         overflowed=[False] * 4)
case("fit_to_bits", "salt_core/tests/test_fixed_point.py:133-138",
     x=[9], total=4, mode="wrap", expected=[-7], overflowed=[True])
case("fit_to_bits", "salt_core/tests/test_fixed_point.py:141-145",
     x=[-9], total=4, mode="wrap", expected=[7], overflowed=[True])
case("fit_to_bits", "salt_core/tests/test_fixed_point.py:148-153",
     x=[9, -9, 100], total=4, mode="saturate", expected=[7, -8, 7],
     overflowed=[True, True, True])

# ---------------------------------------------------------------- one event update
E = "salt_core/tests/test_quant_scan.py"
case("process_event", f"{E}:114-120", v0=0, a=999, ident=True, q=9, vth=100, f_a=4, f_V=0,
     i_V=4, round="round", overflow="wrap", v_final=-7, spiked=False, overflowed=True,
     v_unfitted=9)
case("process_event", f"{E}:136-148", v0=40, a=12, ident=False, q=5, vth=100, f_a=4, f_V=2,
     i_V=8, round="round", overflow="wrap", v_final=50, spiked=False, overflowed=False)
case("process_event", f"{E}:151-156", v0=40, a=12, ident=False, q=5, vth=40, f_a=4, f_V=2,
     i_V=8, round="round", overflow="wrap", v_final=0, spiked=True)
case("process_event", f"{E}:159-167", v0=17, a=999, ident=True, q=3, vth=100, f_a=4, f_V=2,
     i_V=8, round="round", overflow="wrap", v_final=29, overflowed=False)
case("process_event", f"{E}:170-181", v0=7, a=1, ident=False, q=0, vth=100, f_a=2, f_V=0,
     i_V=8, round="round", overflow="wrap", v_final=2)
case("process_event", f"{E}:170-181", v0=7, a=1, ident=False, q=0, vth=100, f_a=2, f_V=0,
     i_V=8, round="truncate", overflow="wrap", v_final=1)
case("process_event", f"{E}:184-193", v0=-6, a=1, ident=False, q=0, vth=100, f_a=2, f_V=0,
     i_V=8, round="round", overflow="wrap", v_final=-1)
case("process_event", f"{E}:184-193", v0=-6, a=1, ident=False, q=0, vth=100, f_a=2, f_V=0,
     i_V=8, round="truncate", overflow="wrap", v_final=-2)
case("process_event", f"{E}:196-209", v0=7, a=999, ident=True, q=1, vth=5, f_a=4, f_V=0, i_V=4,
     round="round", overflow="wrap", v_final=-8, spiked=False, overflowed=True)
case("process_event", f"{E}:212-219", v0=7, a=999, ident=True, q=1, vth=5, f_a=4, f_V=0, i_V=4,
     round="round", overflow="saturate", v_final=0, spiked=True, overflowed=True)
case("process_event", f"{E}:222-227", v0=100, a=999, ident=True, q=50, vth=None, f_a=4, f_V=0,
     i_V=16, round="round", overflow="wrap", v_final=150, spiked=False)
case("process_event", f"{E}:230-235", v0=100, a=1, ident=False, q=1, vth=10 ** 8, f_a=15,
     f_V=14, i_V=16, round="round", overflow="wrap", overflowed=False)
SPEC = "docs/量化模型推論.md"
# spec worked examples: conv2 neuron, f_a=6, f_V=0, register width 11, v_th 35
case("process_event", f"{SPEC}:147-153", v0=-300, a=53, ident=False, q=20, vth=35, f_a=6,
     f_V=0, i_V=11, round="round", overflow="saturate", v_final=-228, spiked=False,
     v_unfitted=-228)
case("process_event", f"{SPEC}:155-160", v0=20, a=56, ident=False, q=25, vth=35, f_a=6,
     f_V=0, i_V=11, round="round", overflow="saturate", v_final=0, spiked=True, v_unfitted=43)
case("process_event", f"{SPEC}:162-169", v0=-1000, a=0, ident=True, q=-63, vth=35, f_a=6,
     f_V=0, i_V=11, round="round", overflow="saturate", v_final=-1024, spiked=False,
     overflowed=True, v_unfitted=-1063)
case("process_event", f"{SPEC}:162-169", v0=-1000, a=0, ident=True, q=-63, vth=35, f_a=6,
     f_V=0, i_V=11, round="round", overflow="wrap", v_final=0, spiked=True, overflowed=True,
     v_unfitted=-1063)
case("process_event", f"{SPEC}:171-175", v0=-300, a=0, ident=False, q=17, vth=35, f_a=6,
     f_V=0, i_V=11, round="round", overflow="saturate", v_final=17, v_unfitted=17)

# ---------------------------------------------------------------- whole queues (run_layer)
case("run_layer", f"{E}:11-26", a=[[999, 12]], ident=[[True, False]], q=[[5, 3]], vth=[100],
     f_a=4, f_V=2, i_V=8, v_final=[27], spike_mask=[[False, False]],
     overflowed=[[False, False]])
case("run_layer", f"{E}:29-46", a=[[14, 13, 0]], ident=[[False, False, True]], q=[[5, 0, 0]],
     vth=[100000], f_a=4, f_V=4, i_V=16, v_final=[65])
case("run_layer", f"{E}:62-75", a=[[999], [999]], ident=[[True], [True]], q=[[20], [20]],
     vth=[15, 25], f_a=4, f_V=0, i_V=8, v_final=[0, 20], spike_mask=[[True], [False]])
case("run_layer", f"{E}:78-90", a=[[999]], ident=[[True]], q=[[9]], vth=[100], f_a=4, f_V=0,
     i_V=4, v_final=[-7], spike_mask=[[False]], overflowed=[[True]])
case("run_layer", f"{E}:93-111", a=[[999, 999], [999, 999]],
     ident=[[True, True], [True, True]], q=[[20, -3], [-30, -5]], vth=[15, 100], f_a=4, f_V=0,
     i_V=6, v_final=[-3, 29], v_unfitted_max=[20, 0], v_unfitted_min=[-3, -35],
     overflowed=[[False, False], [False, True]])

# ---------------------------------------------------------------- decay table
C = "salt_core/tests/test_quant_codes.py"
case("decay_table", f"{C}:61-67", f_a=4, tau=4.0, prefix=[12, 9, 7])
case("decay_table", f"{C}:70-74", f_a=4, tau=64.0, prefix=[15])
case("apply_decay", f"{C}:84-92", f_a=4, tau=4.0, delta_t=[0.0, 1.0, 2.0, 3.0, 60.0],
     is_identity=[True, False, False, False, False], a_tail=[12, 9, 7, 0])

# ---------------------------------------------------------------- queue construction / streams
Q = "salt_core/tests/test_conv_queue.py"
case("compress", f"{Q}:47-80", n_flat=[5, 8, 5, 7, 6, 8, 5, 6], j_flat=[0, 0, 1, 1, 2, 2, 3, 3],
     n_out_spatial=8, max_queue_len=3, n_events=4,
     rows={"5": [0, 1, 3], "6": [2, 3, 4], "7": [1, 4, 4], "0": [4, 4, 4], "1": [4, 4, 4],
           "2": [4, 4, 4], "3": [4, 4, 4], "4": [4, 4, 4]},
     n_real=[0, 0, 0, 0, 0, 3, 2, 1])
case("delta_t_regimes", f"{Q}:97-146", t_gathered=[[1.0, 2.0, 5.0], [3.0, 5.0, 5.0],
                                                    [2.0, 2.0, 2.0]],
     n_real=[3, 2, 1], global_last=5.0, expected=[[1, 1, 3], [3, 2, 0], [2, 3, 0]])
SC = "salt_core/tests/test_stream_conv.py"
case("extract_conv", f"{SC}:30-66", spike_mask=[[True], [False], [True]],
     spike_event_idx=[[2], [0], [0]], event_times=[1.0, 2.0, 3.0, 5.0],
     local_to_global_j=[[0, 1, 3], [2, 3, 4], [1, 4, 4]], max_total_spikes=4,
     n_real=2, src_prefix=[2, 0], times_prefix=[2.0, 5.0], pad_times_above=1e6)
case("extract_conv", f"{SC}:73-95", spike_mask=[[True], [False], [True]],
     spike_event_idx=[[0], [0], [0]], event_times=[10.0, 20.0, 30.0, 40.0, 50.0, 60.0],
     local_to_global_j=[[5], [6], [5]], max_total_spikes=4, n_real=2, src_prefix=[0, 2],
     times_prefix=[60.0, 60.0], pad_times_above=1e6)

# ---------------------------------------------------------------- layers (QuantBackend)
B = "salt_core/tests/test_quant_backend.py"
case("fc_layer", f"{B}:61-74", n_in=1, n_out=2, tau=4.0, q=[[7], [3]], f_a=4, f_V=0, i_V=16,
     vth=[100, 100], times=[0.0], src=[0], n_real=1, max_out_spikes=8, v_final=[7, 3],
     spike_count=0)
case("fc_layer", f"{B}:77-102", n_in=2, n_out=2, tau=4.0, q=[[5, 3], [2, 1]], f_a=4, f_V=0,
     i_V=16, vth=[8, 8], times=[1.0, 2.0, 4.0], src=[0, 1, 0], n_real=3, max_out_spikes=8,
     v_final=[0, 4], spike_count=1)
case("fc_layer", f"{B}:291-302", n_in=1, n_out=1, tau=4.0, q=[[9]], f_a=4, f_V=0, i_V=4,
     vth=None, times=[0.0], src=[0], n_real=1, max_out_spikes=1, v_final=[-7])
case("fc_layer", f"{B}:291-302", n_in=1, n_out=1, tau=4.0, q=[[9]], f_a=4, f_V=0, i_V=4,
     vth=None, overflow="saturate", times=[0.0], src=[0], n_real=1, max_out_spikes=1,
     v_final=[7])
case("fc_layer", f"{B}:257-273", n_in=1, n_out=2, tau=4.0, q=[[50], [45]], f_a=4, f_V=1,
     i_V=16, vth=None, times=[0.0], src=[0], n_real=1, max_out_spikes=1, v_final=[100, 90],
     scale=[1.0, 2.0], readout=[50.0, 90.0])
case("conv_layer", f"{B}:122-140", ic=1, h_in=1, w_in=2, oc=1, k=1, s=1, p=0, tau=16.0,
     max_queue_len=2, max_out_spikes=2, q=[[[[5]]]], f_a=4, f_V=4, i_V=16, vth=[100000],
     times=[2.0, 5.0], src=[0, 1], n_real=2, v_final=[65, 80])
case("conv_layer", f"{B}:226-241", ic=1, h_in=3, w_in=3, oc=1, k=3, s=1, p=0, tau=4.0,
     max_queue_len=4, max_out_spikes=9, q="ones", f_a=8, f_V=2, i_V=16, vth=[1000],
     times=[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0, 9.0], src=[0, 1, 2, 3, 4, 5, 6, 7, 8],
     n_real=9, needed_queue=10, fits=False)
case("conv_layer", f"{B}:226-241", ic=1, h_in=3, w_in=3, oc=1, k=3, s=1, p=0, tau=4.0,
     max_queue_len=10, max_out_spikes=9, q="ones", f_a=8, f_V=2, i_V=16, vth=[1000],
     times=[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0, 9.0], src=[0, 1, 2, 3, 4, 5, 6, 7, 8],
     n_real=9, needed_queue=10, fits=True)
case("conv_layer", f"{B}:244-254", ic=1, h_in=3, w_in=3, oc=1, k=3, s=1, p=0, tau=4.0,
     max_queue_len=10, max_out_spikes=2, q="ones", f_a=8, f_V=0, i_V=16, vth=[1],
     times=[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0, 9.0], src=[0, 1, 2, 3, 4, 5, 6, 7, 8],
     n_real=9, spike_count=9, fits=False)
case("conv_layer", f"{B}:244-254", ic=1, h_in=3, w_in=3, oc=1, k=3, s=1, p=0, tau=4.0,
     max_queue_len=10, max_out_spikes=9, q="ones", f_a=8, f_V=0, i_V=16, vth=[1],
     times=[1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0, 9.0], src=[0, 1, 2, 3, 4, 5, 6, 7, 8],
     n_real=9, spike_count=9, fits=True)
# Tie order of the output stream (salt_core/tests/test_stream_tiebreak.py:31-70 states it for the
# float backend; the same extract_output_events_fc orders the integer path).  Hand computation:
# two events at t=1 from inputs 0 and 1 (identity decay); neuron 0 (q=[6, 6]) reaches 12 >= 10
# at event 1, neuron 1 (q=[12, 0]) fires at event 0 and then stays at 0, so the stream is
# [neuron 1, neuron 0] although both spikes share the timestamp.
case("fc_layer", "salt_core/tests/test_stream_tiebreak.py:31-70 (integer restatement)",
     n_in=2, n_out=2, tau=4.0, q=[[6, 6], [12, 0]], f_a=4, f_V=0, i_V=16, vth=[10, 10],
     times=[1.0, 1.0], src=[0, 1], n_real=2, max_out_spikes=4, v_final=[0, 0],
     spike_count=2, src_prefix=[1, 0], times_prefix=[1.0, 1.0])

# ---------------------------------------------------------------- float chunked scan (FC)
F = "salt_core/tests/test_fc_forward.py"
# test_fc_forward.py:1-13 hand example (docs/math/全連接forward訓練範例.md): b1 fires once at
# global event 2 and resets; b2 never fires and ends at 0.539.  The result must not depend on
# chunk_size (1 or the whole stream); max_steps = n_real_events.
for chunk, extra in ((1, 0), (3, 2)):
    case("float_fc_layer", f"{F}:30-64 (chunk_size={chunk})", n_in=2, n_out=2, tau=4.0,
         v_th=1.0, w=[[0.6, 0.5], [0.3, 0.2]], times=[1.0, 2.0, 4.0], src=[0, 1, 0], n_real=3,
         chunk_size=chunk, max_extra_steps=extra, max_out_spikes=6, v_final=[0.0, 0.539],
         v_tol=1e-4, spikes_per_neuron=[[2], []])
# test_fc_layer.py:17-55: one neuron, inputs 0 (w=1.0, fires alone) and 1 (w=0.1), events at
# 0..9 ms with input 0 at events 0 and 5.  chunk 5 needs 3 steps (1, 5, 4 events) but gets 2:
# extra-steps need 2 (b>0: 10 events, energy floor(2.8/1)=2, m*=2, bound 2+ceil(8/5)=4, base 2).
# With enough steps every event is used and V matches chunk_size=1: after the reset at event 5,
# four events of 0.1 with Δt=1 (a=15/16): 0.1, 0.19375, 0.281640625, 0.36403808...
T = "salt_core/tests/test_fc_layer.py"
TWO = dict(n_in=2, n_out=1, tau=16.0, v_th=1.0, w=[[1.0, 0.1]],
           times=[float(i) for i in range(10)], src=[0, 1, 1, 1, 1, 0, 1, 1, 1, 1], n_real=10)
case("float_fc_layer", f"{T}:33-43", chunk_size=5, max_extra_steps=0, max_out_spikes=8192,
     fits=False, extra_steps_needed=2, v_final_differs=[0.36403808], **TWO)
case("float_fc_layer", f"{T}:46-55", chunk_size=5, max_extra_steps=2, max_out_spikes=8192,
     fits=True, spike_count=2, v_final=[0.36403808], v_tol=1e-6, **TWO)
case("float_fc_layer", f"{T}:46-55 (chunk_size=1)", chunk_size=1, max_extra_steps=0,
     max_out_spikes=8192, fits=True, spike_count=2, v_final=[0.36403808], v_tol=1e-6, **TWO)
case("float_fc_layer", f"{T}:58-65", chunk_size=1, max_extra_steps=0, max_out_spikes=1,
     fits=False, n_real_out=2, **TWO)
case("float_fc_layer", f"{T}:58-65 (roomy)", chunk_size=1, max_extra_steps=0, max_out_spikes=2,
     fits=True, n_real_out=2, **TWO)
# test_stream_tiebreak.py: same-timestamp spikes leave in global event order, not neuron order;
# chunk_size = stream length and max_steps = 1, so a neuron stops after its first spike.
S = "salt_core/tests/test_stream_tiebreak.py"
case("float_fc_layer", f"{S}:31-70", n_in=1, n_out=2, tau=4.0, v_th=1.0, w=[[0.6], [1.2]],
     times=[1.0, 1.0], src=[0, 0], n_real=2, chunk_size=2, max_extra_steps=0, max_out_spikes=4,
     spikes_per_neuron=[[1], [0]], src_prefix=[1, 0], times_prefix=[1.0, 1.0], n_real_out=2)
case("float_fc_layer", f"{S}:73-111", n_in=1, n_out=3, tau=4.0, v_th=1.0,
     w=[[0.4], [1.2], [0.6]], times=[1.0, 1.0, 1.0], src=[0, 0, 0], n_real=3, chunk_size=3,
     max_extra_steps=0, max_out_spikes=6, spikes_per_neuron=[[2], [0], [1]],
     src_prefix=[1, 2, 0], times_prefix=[1.0, 1.0, 1.0], n_real_out=3)
# test_affine.py:21-49: the composed prefix maps equal the sequential h = V*a + w (1e-6).
case("affine_scan", "salt_core/tests/test_affine.py:21-49", tau=16.0, v0=0.37,
     n_ms=[0, 2, 1, 5, 0, 3], w=[0.3, -0.1, 0.5, 0.2, 0.05, -0.2], tol=1e-6)

if __name__ == "__main__":
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "known_answers.json")
    with open(out, "w") as f:
        json.dump(CASES, f, indent=1, ensure_ascii=False)
    print(f"wrote {len(CASES)} cases to {out}")
