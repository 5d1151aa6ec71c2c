"""Path-loading of the reference's own logits processors.

TEST INFRASTRUCTURE / CPU BASELINE ONLY: used by tests/golden/make_golden.py
(fixtures) and by bench.py's reference arm and CPU-baseline leg (which time
the reference's own processors on the host cores).  Nothing in the product
package imports it.

The reference's package ``__init__`` files import dependencies the processor
modules do not need, so the package roots are stubbed with ``__path__``
pointing into the reference tree -- the recipe of the reference's own tests
(tests/test_logit_processors.py:11-29) -- and only these modules execute:

  osuT5/osuT5/event.py
  osuT5/osuT5/inference/logit_processors.py          (build_logits_processor_list)
  osuT5/osuT5/inference/optimized/single/logits.py   (stateful monotonic processor)
  osuT5/osuT5/inference/compiled_decode.py: _sample  (compiled from its AST alone)

``dataset.data_utils`` and ``tokenizer`` are replaced by the two constants the
processors read (TIMED_EVENTS, its member names read from data_utils.py's
source; MILISECONDS_PER_STEP); the tokenizer object is duck-typed as in the
reference's tests (``_FakeTokenizer``).
"""

from __future__ import annotations

import ast
import sys
import types
from pathlib import Path


def _stub_pkg(name: str, path: Path) -> None:
    mod = types.ModuleType(name)
    mod.__path__ = [str(path)]
    sys.modules[name] = mod


def load_reference(ref: Path):
    """(event module, logit_processors module, optimized.single.logits module,
    the AST module of compiled_decode._sample) from the reference tree `ref`."""
    ref = Path(ref)
    if not (ref / "osuT5" / "osuT5" / "inference" / "logit_processors.py").exists():
        raise FileNotFoundError(f"no reference processors under {ref}")
    _stub_pkg("osuT5", ref / "osuT5")
    _stub_pkg("osuT5.osuT5", ref / "osuT5" / "osuT5")
    _stub_pkg("osuT5.osuT5.inference", ref / "osuT5" / "osuT5" / "inference")
    _stub_pkg("osuT5.osuT5.inference.optimized", ref / "osuT5" / "osuT5" / "inference" / "optimized")
    _stub_pkg("osuT5.osuT5.inference.optimized.single", ref / "osuT5" / "osuT5" / "inference" / "optimized" / "single")
    _stub_pkg("osuT5.osuT5.dataset", ref / "osuT5" / "osuT5" / "dataset")
    du = types.ModuleType("osuT5.osuT5.dataset.data_utils")
    du.TIMED_EVENTS = []
    sys.modules[du.__name__] = du
    tk = types.ModuleType("osuT5.osuT5.tokenizer")
    tk.MILISECONDS_PER_STEP = 10
    tk.Tokenizer = object
    sys.modules[tk.__name__] = tk
    import osuT5.osuT5.event as ev

    du.TIMED_EVENTS[:] = [ev.EventType[n] for n in timed_event_names(ref)]
    import osuT5.osuT5.inference.logit_processors as lp
    import osuT5.osuT5.inference.optimized.single.logits as sl

    src = (ref / "osuT5" / "osuT5" / "inference" / "compiled_decode.py").read_text()
    tree = ast.parse(src)
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "_sample")
    return ev, lp, sl, ast.Module(body=[fn], type_ignores=[])


def timed_event_names(ref: Path) -> list:
    """Member names of data_utils.TIMED_EVENTS, read from the reference source
    (osuT5/osuT5/dataset/data_utils.py) without importing the module."""
    src = (Path(ref) / "osuT5" / "osuT5" / "dataset" / "data_utils.py").read_text()
    for node in ast.parse(src).body:
        if isinstance(node, ast.Assign) and any(getattr(t, "id", None) == "TIMED_EVENTS" for t in node.targets):
            return [e.attr for e in node.value.elts]
    raise LookupError("TIMED_EVENTS not found in data_utils.py")


def make_tokenizer(ev, *, ts=(16, 116), sos=1, context_sos=None, extra=None, context_eos=None, ts_min=0,
                   vocab=None):
    """Duck-typed tokenizer with the attributes the processors read; encode()
    follows tokenizer.py:276-290 (first id + value - min_value)."""

    class Tok:
        def encode(self, event):
            er = self.event_range[event.type]
            if not er.min_value <= event.value <= er.max_value:
                raise ValueError(f"event value {event.value} out of range")
            return self.event_start[event.type] + event.value - er.min_value

    t = Tok()
    t.sos_id = sos
    t.eos_id = 2
    t.context_sos = dict(context_sos or {})
    t.context_eos = dict(context_eos or {})
    t.event_start = {ev.EventType.TIME_SHIFT: ts[0]}
    t.event_end = {ev.EventType.TIME_SHIFT: ts[1]}
    t.event_range = {ev.EventType.TIME_SHIFT: types.SimpleNamespace(min_value=ts_min,
                                                                     max_value=ts_min + ts[1] - ts[0] - 1)}
    t.vocab_size_out = vocab
    for name, (a, b) in (extra or {}).items():
        t.event_start[ev.EventType[name]] = a
        t.event_end[ev.EventType[name]] = b
    return t
