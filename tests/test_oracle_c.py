"""The C restatement (oracle/gdn_oracle.c) against the numpy oracle.  CPU only."""
import numpy as np

import gdn_oracle as O


def test_c_oracle_matches_numpy_oracle_with_gqa_and_states():
    rng = np.random.default_rng(21)
    inp = O.synth_decode_inputs(rng, 2, 3, Hk=2, Hv=6)
    states = np.empty((2, 6, 3, 128, 128), np.float32)
    o, S = O.recurrent_c(inp["q"], inp["k"], inp["v"], inp["a"], inp["b"], inp["A_log"], inp["dt_bias"],
                         inp["S0"], states=states, nthreads=2)
    al, bt = O.gates(inp["a"], inp["b"], inp["A_log"], inp["dt_bias"])
    ro, rS, rst = O.delta_reference(O.expand_heads(inp["q"], 6), O.expand_heads(inp["k"], 6), inp["v"],
                                    al, bt, inp["S0"], collect=True)
    assert O.rel_err(o, ro) < 1e-5 and O.rel_err(S, rS) < 1e-5 and O.rel_err(states, rst) < 1e-5


def test_c_oracle_in_place_and_zero_state():
    rng = np.random.default_rng(22)
    inp = O.synth_decode_inputs(rng, 1, 2, Hk=1, Hv=3)
    S = inp["S0"].copy()
    O.recurrent_c(inp["q"], inp["k"], inp["v"], inp["a"], inp["b"], inp["A_log"], inp["dt_bias"], S, S_out=S)
    al, bt = O.gates(inp["a"], inp["b"], inp["A_log"], inp["dt_bias"])
    args = (O.expand_heads(inp["q"], 3), O.expand_heads(inp["k"], 3), inp["v"], al, bt)
    _, rS = O.delta_reference(*args, inp["S0"])
    assert O.rel_err(S, rS) < 1e-5
    o, S0 = O.recurrent_c(inp["q"], inp["k"], inp["v"], inp["a"], inp["b"], inp["A_log"], inp["dt_bias"])
    ro, rS = O.delta_reference(*args)
    assert O.rel_err(o, ro) < 1e-5 and O.rel_err(S0, rS) < 1e-5
