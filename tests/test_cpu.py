"""CPU tests (no GPU): the C-ABI library loads and exports every declared entry point; the host task compiler's atom
layout equals the reference's dense layout; the oracle reproduces the reference's golden vectors; generators are
deterministic."""

import hashlib
import re
import os
from pathlib import Path

import numpy as np
import pytest

from mymyr_b200 import _lib, tasks
from mymyr_b200.task import Task

ROOT = Path(__file__).resolve().parent.parent
# the reference checkout (read-only; present where the oracle is built, absent on GPU boxes)
REF_TASKS = Path(os.environ.get("MYMYR_REFERENCE", Path(__file__).resolve().parents[2] / "reference")) / "tests" / "data" / "tasks"


def declared_symbols():
    text = (ROOT / "include" / "mymyr_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b2_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)
    assert b"sm_100a" in L.b2_version()


def _reference_keywords(source: Path, name: str) -> list[tuple[str, str | None]]:
    """The keyword arguments ("x"_a or "x"_a = default) of m.def("<name>", ...) in a nanobind source, in order."""
    text = source.read_text()
    seg = text[re.search(r'm\.def\(\s*"' + name + r'",', text).end():]
    seg = seg[re.search(r'"[a-z_]+"_a', seg).start():]
    seg = seg[: seg.index('");')]
    return [(k, v.strip() if v else None) for k, v in re.findall(r'"([a-z_]+)"_a(?:\s*=\s*([^,)]+))?', seg)]


def test_brfs_keywords_match_the_reference_binding():
    """cuda.brfs takes the keywords of the reference's mymyr.cuda.brfs with its defaults (extra keywords follow)."""
    import inspect

    src = REF_TASKS.parents[2] / "python" / "src" / "cuda_bindings.cpp"
    if not src.exists():
        pytest.skip("reference checkout absent")
    from mymyr_b200 import cuda as b2cuda

    ref_kw = _reference_keywords(src, "brfs")
    assert [k for k, _ in ref_kw][:3] == ["task", "ctx", "witness_pruning"]
    sig = inspect.signature(b2cuda.brfs).parameters
    ours = list(sig)
    assert ours[: len(ref_kw)] == [k for k, _ in ref_kw]
    convert = {"true": True, "false": False, "nb::none(": None}  # the default up to its first comma or ")"
    for k, d in ref_kw:
        if d is not None:
            assert sig[k].default == convert[d], (k, d, sig[k].default)
        if k != "task":
            assert sig[k].kind is inspect.Parameter.KEYWORD_ONLY, k


def test_errors_cross_the_abi_as_status_codes():
    with pytest.raises(RuntimeError, match="task text"):
        Task.from_text("O 2\nP 1\nF 1 p\nSI 0\nFI 1\n0 5\n", host_only=True)  # object out of range
    with pytest.raises(ValueError, match="does not support|does not run"):
        Task.from_text("O 1\nP 1\nD 1 p\nSI 0\nFI 0\nG 0\nA 0\n", host_only=True)


GENERATED = {
    "tower7": lambda: tasks.tower(7, 0),
    "tower5_s3": lambda: tasks.tower(5, 3),
    "transport": lambda: tasks.transport(2, 40, 2, 0),
    "transport_3_4_1": lambda: tasks.transport(3, 4, 1, 2),
    "tile4x4": lambda: tasks.sliding_tile(4, 4, 60, 0),
    "tile3x3": lambda: tasks.sliding_tile(3, 3, 40, 5),
    "random0": lambda: tasks.random_domain(0),
    "random1": lambda: tasks.random_domain(1),
    "counters": lambda: tasks.counters(3, 5, 0),
}


def test_generators_are_deterministic_and_pinned():
    digests = {k: hashlib.sha256(f().encode()).hexdigest()[:16] for k, f in GENERATED.items()}
    again = {k: hashlib.sha256(f().encode()).hexdigest()[:16] for k, f in GENERATED.items()}
    assert digests == again
    pinned = (ROOT / "tests" / "golden" / "task_digests.txt")
    want = dict(line.split() for line in pinned.read_text().splitlines() if line.strip())
    assert digests == want


@pytest.mark.parametrize("name", ["tile4x4", "transport_2_200_3", "counters"])
def test_compiled_matcher_kernels_build_on_the_host(name):
    """The task's generated matcher and the kernels over it (count, expand, fused expand + push, env, batched expand)
    compile for sm_100a with NVRTC without a device."""
    text = {"tile4x4": tasks.sliding_tile(4, 4, 60, 0), "transport_2_200_3": tasks.transport(2, 200, 3, 0),
            "counters": tasks.counters(3, 5, 0)}[name]
    src = Task.from_text(text, host_only=True).compile()
    assert "b2::gen" in src or "namespace" in src


def test_bench_config_shapes():
    t = Task.from_text(tasks.sliding_tile(4, 4, 60, 0), host_only=True)
    assert (t.words, t.fluent_slots, t.num_objects) == (4, 256, 31)
    t = Task.from_text(tasks.tower(7, 0), host_only=True)
    assert (t.words, t.fluent_slots) == (2, 71)
    t = Task.from_text(tasks.transport(2, 40, 2, 0), host_only=True)
    assert (t.words, t.fluent_slots) == (3, 164)


@pytest.mark.parametrize("name", sorted(GENERATED))
def test_layout_matches_reference_dense(ref, name):
    text = GENERATED[name]()
    rt = ref.RefTask(text, atoms="dense")
    t = Task.from_text(text, host_only=True)
    assert (t.words, t.fluent_slots) == (rt.words, rt.fluent_slots)
    assert np.array_equal(t.initial_state(), rt.initial_state())


def _suite_texts():
    if not REF_TASKS.exists():
        return []
    return sorted(REF_TASKS.glob("*.txt"))


@pytest.mark.parametrize("path", _suite_texts(), ids=lambda p: p.stem)
def test_layout_matches_reference_on_suite(ref, path):
    """The reference's own task fixtures (read in place; not copied): dense layouts agree wherever the device path
    accepts the task."""
    text = path.read_text()
    try:
        t = Task.from_text(text, host_only=True)
    except ValueError as e:
        pytest.skip(f"unsupported on the device path: {e}")
    rt = ref.RefTask(text, atoms="dense")
    assert (t.words, t.fluent_slots) == (rt.words, rt.fluent_slots)
    assert np.array_equal(t.initial_state(), rt.initial_state())


# golden counts of exhaustive BrFS (witness pruning on), tests/cpp/support/suite.hpp:31-54 of the reference
SUITE_GOLDEN = {
    "gripper__prob05": (376832, 2031616, 2),
    "depot__p02": (40320, 376560, 9),
    "pegsol-08-strips__p22": (99457, 189967, 2),
    "philosophers__p03-phil4": (47938, 121820, 1),
    "organic-synthesis-opt18-strips__p20": (41311, 52548, 24),
    "openstacks-opt08-adl__p03": (97953, 548161, 6),
}


@pytest.mark.parametrize("name", sorted(SUITE_GOLDEN))
def test_oracle_reproduces_suite_golden_counts(ref, name):
    path = REF_TASKS / f"{name}.txt"
    if not path.exists():
        pytest.skip("reference fixtures absent")
    r = ref.RefTask(path.read_text(), atoms="auto").brfs(threads=1, stop_at_goal=False)
    assert (r["states"], r["generated"], r["num_goal_states"]) == SUITE_GOLDEN[name]


def test_oracle_philox_known_answers(ref):
    """Random123 philox4x32-10 known answers (tests/cpp/rl/test_env.cpp:167-194 of the reference)."""
    import ctypes as C

    kats = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
            ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
            ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
             (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    out = np.zeros(4, np.uint32)
    for ctr, key, want in kats:
        ref.lib().ref_philox_block(*ctr, *key, out.ctypes.data)
        assert tuple(int(x) for x in out) == want


def test_tile_brfs_golden_file_matches_reference(ref):
    """The golden BrFS results the bench checks its searches against equal the reference's own BrFS (shallow depths;
    the generating script, tests/golden/make_brfs_golden.py, writes every depth the same way)."""
    import json

    from mymyr_b200 import tasks

    g = json.loads((ROOT / "tests" / "golden" / "tile4x4_brfs.json").read_text())["depths"]
    assert all(str(d) in g for d in range(12, 26))
    rt = ref.RefTask(tasks.sliding_tile(4, 4, 60, 0))
    for d in (12, 15, 18):
        r = rt.brfs(threads=4, max_depth=d, stop_at_goal=False, fingerprint=True, store="concurrent")
        assert g[str(d)]["states"] == r["states"] and g[str(d)]["fingerprint"] == f"{r['fingerprint']:#018x}"
        assert g[str(d)]["layer_counts"] == [list(x) for x in r["layer_counts"]]


@pytest.mark.parametrize("atoms", ["auto", "reachable", "dense"])
@pytest.mark.parametrize("name", ["tower7", "transport", "tile4x4", "counters", "random0"])
def test_reference_side_shim_describes_the_task(ref, name, atoms):
    """The reference-side shim (include/mymyr_b200_shim.hpp, compiled against the reference's headers by
    oracle/Makefile): describe() of a reference Task's TaskData gives a device task whose words, fluent slots and
    initial row equal the reference's dense twin of the task (Task::translate for Auto and Reachable slots)."""
    if not ref.shim_available():
        pytest.skip("oracle/_ref/libshim_check.so not built")
    rc, msg = ref.shim_layout(GENERATED[name](), atoms)
    assert rc == 0, msg


@pytest.mark.parametrize("path", _suite_texts()[:8], ids=lambda p: p.stem)
def test_reference_side_shim_on_suite_tasks(ref, path):
    """The shim on the reference's own task fixtures (read in place): a task the device path accepts is described
    with the reference's dense layout; one it does not is refused with std::invalid_argument."""
    if not ref.shim_available():
        pytest.skip("oracle/_ref/libshim_check.so not built")
    rc, msg = ref.shim_layout(path.read_text(), "auto")
    assert rc == 0 or (rc == -1 and ("support" in msg or "does not run" in msg)), msg
