"""Host-side checks of the benchmark presets and the model-config mirror (no
GPU): every preset leaves room after its prompt for the tokens it generates
and for the positions bench.py's default run reaches (positions at or past
max_context are not stored), and the Python config converts field by field
to the C struct the engine takes."""
import pytest

import pocketforge_b200 as pf
from pocketforge_b200 import _lib


@pytest.mark.parametrize("name", sorted(pf.PRESETS))
def test_preset_leaves_room_after_the_prompt(name):
    pr = pf.PRESETS[name]
    m = pr["model"]
    rows = m.n_mtp_heads + 1  # one verify batch in flight
    assert pr["prompt"] + pr["gen"] + rows <= m.max_context, name
    # bench.py's default run: W = 4 warm-up + 64 timed steps, two spare steps, 8 spare positions
    assert pr["prompt"] + (4 + 64 + 2) * rows + 8 <= m.max_context, name
    assert pr["seqs"] >= 1 and 1 <= m.n_mtp_heads <= 8
    assert m.sink_size + m.window_size > 0 and m.pool_block > 0


@pytest.mark.parametrize("name", sorted(pf.PRESETS))
def test_model_config_converts_field_by_field(name):
    m = pf.PRESETS[name]["model"]
    c = m.to_c()
    for field, _ in _lib.ModelConfigC._fields_:
        if field == "qtype":
            assert [c.qtype[i] for i in range(7)] == [int(q) for q in m.qtype]
        elif isinstance(getattr(m, field), float):
            assert getattr(c, field) == pytest.approx(getattr(m, field), rel=1e-7)
        else:
            assert getattr(c, field) == int(getattr(m, field)), field
