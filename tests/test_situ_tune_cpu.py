"""The in-situ tuner's selection logic on the host, with a made-up cost model in place of
the stand-in's timing (no GPU needed)."""

from __future__ import annotations

from int8_linear.kernel import Config
from int8_linear.situ_tune import accept, coordinate_pass, layer_options, write_entries

A, B, C, D = (Config(16, 128, split=1), Config(16, 128, split=3, cluster=2),
              Config(128, 256, split=3, cluster=8), Config(32, 128))


def test_layer_options_keep_order_and_drop_repeats():
    assert layer_options(A, B, [B, C, A, D], top=3) == [A, B, C]
    assert layer_options(A, A, [D, C], top=1) == [A, D]


def test_coordinate_pass_keeps_each_linears_fastest_option():
    cost = {("qkv", A): 3.0, ("qkv", B): 2.0, ("qkv", C): 2.5,
            ("o", A): 1.0, ("o", C): 0.5, ("o", D): 0.7}
    calls = []

    def measure(cfgs):
        calls.append(dict(cfgs))
        return sum(cost[(name, cfg)] for name, cfg in cfgs.items())

    chosen, trials = coordinate_pass({"qkv": A, "o": A}, {"qkv": [A, B, C], "o": [A, C, D]}, measure)
    assert chosen == {"qkv": B, "o": C}
    assert len(trials) == 6 and trials[0] == ("qkv", A, 4.0)
    # the second linear is tried with the first already at its best
    assert all(c["qkv"] == B for c in calls[3:])


def test_coordinate_pass_sees_interactions_between_linears():
    """A tiling that is fastest alone can lose next to its neighbour's tiling: the pass
    measures each option in the whole step, so the interaction decides."""
    def measure(cfgs):
        base = {A: 2.0, C: 1.5}[cfgs["qkv"]] + {A: 2.0, C: 1.5}[cfgs["o"]]
        return base + (1.0 if cfgs["qkv"] == C and cfgs["o"] == C else 0.0)

    chosen, _ = coordinate_pass({"qkv": A, "o": A}, {"qkv": [A, C], "o": [A, C]}, measure)
    assert chosen == {"qkv": C, "o": A}


def test_accept_needs_a_one_percent_gain():
    assert accept(40.0, 39.5)
    assert not accept(40.0, 39.7)
    assert not accept(40.0, 41.0)


def test_written_entries_read_back_as_configs():
    table = {}
    write_entries(table, {"qkv_proj": (2048, 4096), "o_proj": (2048, 2048)}, 4,
                  {"qkv_proj": C, "o_proj": B}, 38.12345)
    assert Config(**table["2048x4096"]["4"]["config"]) == C
    assert Config(**table["2048x2048"]["4"]["config"]) == B
    assert table["2048x2048"]["4"]["stand_in_us"] == 38.123
