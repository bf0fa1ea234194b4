"""A tile graph's specialised kernel on the CPU: its source is the lowered
program as compile-time constants (one entry per device instruction, one
descriptor per window), and NVRTC compiles it for sm_100a without a GPU for
every form the launcher can choose (two or four groups per thread, bulk or
direct inputs, a reduction, chained windows). The reference compiles each
graph with NVRTC the same way (tile/run.go:38-41)."""
import re

import numpy as np
import pytest

from simtgo_b200 import tile
from simtgo_b200._lib import SimtgoError
from test_tile_lowering import _chained_graph, _random_graph

f32 = np.float32


def _available():
    return tile.JITInfo()[1]


needs_nvrtc = pytest.mark.skipif(not _available(), reason="libnvrtc cannot be opened")


def twelve(n=4099):
    rng = np.random.default_rng(6)
    g = tile.New()
    a, b, c = (g.Input(rng.uniform(-4, 4, n).astype(f32)) for _ in range(3))
    s = tile.Scale(a, 0.5)
    ab = tile.Abs(b)
    h = np.full(31, 1 / 31, f32)
    return tile.Mul(tile.Hypot(tile.Add(tile.Mul(s, tile.Sqrt(ab)), c), tile.FIR(s, h)), ab)


def test_source_holds_the_program():
    t = twelve()
    n_insn, n_in, n_win = t.ProgramSize()
    src = t.JITSource(groups=4, bulk=True)
    code = src.split("code[] = {", 1)[1].split("};", 1)[0]
    assert len(re.findall(r"\{\d+, \d+, \d+, \d+, \d+, 0\.0f, 0u\}", code)) == n_insn
    fir = src.split("fir[] = {", 1)[1].split("};", 1)[0]
    assert fir.count("{") == n_win == 1
    assert ", 31, " in fir  # the window's taps
    assert "tile_body<true, 4, Spec>" in src
    assert "tile_body<false, 2, Spec>" in t.JITSource(groups=2, bulk=False)
    # SCALE factors and tap values are not in the source: they stay in the
    # parameter block, so graphs that differ only in them share a kernel.
    assert "0.5" not in src and "0.0322" not in src


def test_arguments_refused():
    t = twelve()
    with pytest.raises(SimtgoError):
        t.JITSource(groups=3)
    with pytest.raises(SimtgoError):
        t.JITSource(reduce=7)
    with pytest.raises(SimtgoError):
        tile.SetJIT(3)
    mode = tile.JITInfo()[0]
    tile.SetJIT(0)
    assert tile.JITInfo()[0] == 0
    tile.SetJIT(mode)


@needs_nvrtc
@pytest.mark.parametrize("groups,bulk", [(4, True), (2, True), (4, False), (2, False)])
def test_twelve_node_compiles(groups, bulk):
    twelve().JITSource(groups=groups, bulk=bulk, compile=True)


@needs_nvrtc
@pytest.mark.parametrize("reduce", [0, 3])
def test_reduction_compiles(reduce):
    twelve().JITSource(reduce=reduce, groups=4, compile=True)


@needs_nvrtc
@pytest.mark.parametrize("seed", range(8))
def test_random_graphs_compile(seed):
    """Every form the launcher can pick compiles for random graphs (shared
    values, x-op-x nodes, windows, reductions), one form per seed."""
    root, _ = _random_graph(seed, 3001, 0)
    reduce = (-1, 0, 3, -1)[seed % 4]
    root.JITSource(reduce=reduce, groups=4 if seed % 2 else 2, bulk=seed % 3 != 2,
                   compile=True)


@needs_nvrtc
@pytest.mark.parametrize("seed", [1, 2, 5])
def test_chained_windows_compile(seed):
    root, _ = _chained_graph(seed, 3001, 0)
    root.JITSource(groups=2, bulk=seed != 2, compile=True)


@needs_nvrtc
def test_disk_cache_across_processes(tmp_path):
    """A compiled kernel is kept on disk and a new process takes it from
    there instead of compiling; a corrupted entry is a miss, not a crash."""
    import os
    import subprocess
    import sys

    prog = (
        "import numpy as np\n"
        "from simtgo_b200 import tile\n"
        "g = tile.New()\n"
        "a = g.Input(np.ones(3001, np.float32))\n"
        "t = tile.Add(tile.Scale(a, 2.0), tile.FIR(a, np.full(5, 0.2, np.float32)))\n"
        "t.JITSource(groups=2, bulk=True, compile=True)\n"
        "print(tile.JITInfo()[2], tile.JITInfo()[4])\n")
    env = dict(os.environ, SIMTGO_B200_CACHE=str(tmp_path / "cache"))
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

    def run():
        out = subprocess.run([sys.executable, "-c", prog], env=env, cwd=root, check=True,
                             capture_output=True, text=True).stdout.split()
        return int(out[0]), int(out[1])

    assert run() == (1, 0)          # compiled, written
    files = list((tmp_path / "cache").glob("*.cubin"))
    assert len(files) == 1
    assert run() == (0, 1)          # read back
    data = bytearray(files[0].read_bytes())
    data[20] ^= 0xFF                 # the stored identity no longer matches
    files[0].write_bytes(bytes(data))
    assert run() == (1, 0)          # a miss: compiled again and rewritten
    assert run() == (0, 1)
    files[0].write_bytes(files[0].read_bytes()[:100])  # truncated mid-identity
    assert run() == (1, 0)
    assert run() == (0, 1)
    env["SIMTGO_B200_CACHE"] = "off"
    assert run() == (1, 0)


@needs_nvrtc
@pytest.mark.parametrize("reduce", [0, 1, 2, 3])
def test_streaming_chain_compiles(reduce):
    """The streaming reduction's kernel for a chain on one input: the steps
    in order as constants, the kernel named by its template instance."""
    g = tile.New()
    a = g.Input(np.ones(5000, f32))
    t = tile.Mul(tile.Sqrt(tile.Abs(tile.Scale(a, -2.0))), tile.Sqrt(tile.Abs(tile.Scale(a, -2.0))))
    # Mul of two different nodes is not a chain; a chain is x op x:
    s = tile.Sqrt(tile.Abs(tile.Scale(a, -2.0)))
    c = tile.Add(s, s)
    src = c.JITSource(reduce=reduce, groups=0, compile=True)
    assert "static constexpr int n = 4;" in src
    assert "op[] = {6, 8, 7, 3}" in src                     # Scale, Abs, Sqrt, Add
    assert f"k_red_direct<{reduce}, tilek::StaticChain<Steps>>" in src
    with pytest.raises(SimtgoError):
        t.JITSource(reduce=reduce, groups=0)                 # not a chain
    with pytest.raises(SimtgoError):
        c.JITSource(reduce=-1, groups=0)                     # not a reduction


def test_without_nvrtc(tmp_path):
    """Where libnvrtc cannot be opened, mode 1 reports it unavailable (and
    launches would use the interpreter), and compiling a specialised source
    fails with a message instead of crashing."""
    import os
    import subprocess
    import sys

    prog = (
        "import numpy as np\n"
        "from simtgo_b200 import tile\n"
        "from simtgo_b200._lib import SimtgoError\n"
        "m, avail, _, _, _ = tile.JITInfo()\n"
        "g = tile.New()\n"
        "a = g.Input(np.ones(100, np.float32))\n"
        "t = tile.Scale(a, 2.0)\n"
        "src = t.JITSource(groups=4)\n"
        "try:\n"
        "    t.JITSource(groups=4, compile=True)\n"
        "    print(m, avail, 'compiled')\n"
        "except SimtgoError as e:\n"
        "    print(m, avail, 'refused', 'could not be opened' in str(e))\n")
    env = dict(os.environ, SIMTGO_NVRTC_LIB=str(tmp_path / "no_such_libnvrtc.so"))
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "-c", prog], env=env, cwd=root, check=True,
                         capture_output=True, text=True).stdout.split()
    assert out == ["1", "False", "refused", "True"]


_OPS = {3: "add", 4: "mul", 5: "hypot", 6: "scale", 7: "sqrt", 8: "abs", 9: "firacc"}


def _steps_of(op, flags):
    """The listing's step kinds of one device instruction, decoded from its
    op and flags the way the kernel runs them: load, operation, temporary,
    window tile, output, end."""
    steps = []
    if flags & 1:
        steps.append("lda")
    if op in _OPS:
        steps.append(_OPS[op])
    for bit, name in ((16, "sta"), (32, "stage"), (64, "store"), (128, "end")):
        if flags & bit:
            steps.append(name)
    return steps


@pytest.mark.parametrize("seed", range(6))
def test_source_is_the_listed_program(seed):
    """The specialised source's constant program is the lowered program the
    listing (Tensor.Source) shows, instruction by instruction; main_start and
    the windows' start points agree too."""
    root, _ = _random_graph(seed, 3001, 0)
    listing = [ln for ln in root.Source().splitlines() if ln[:1].isdigit()]
    want = [[st.split()[0] for st in ln.split(" ", 1)[1].split(" | ")] for ln in listing]
    src = root.JITSource(groups=2, bulk=True)
    code = src.split("code[] = {", 1)[1].split("};", 1)[0]
    got = [_steps_of(int(m[0]), int(m[1]))
           for m in re.findall(r"\{(\d+), (\d+), \d+, \d+, \d+, 0\.0f, 0u\}", code)]
    assert got == want
    lines = root.Source().splitlines()
    main = int(re.search(r"main_start = (\d+)", src).group(1))
    assert lines[lines.index("main") + 1].startswith(f"{main} ")
    fir = src.split("fir[] = {", 1)[1].split("};", 1)[0]
    starts = [int(m) for m in re.findall(r"\{(\d+), \d+, \d+, \d+\}", fir)]
    heads = [i for i, ln in enumerate(lines) if ln.startswith("window ")]
    if heads:
        assert [int(lines[i + 1].split()[0]) for i in heads] == starts
        assert [int(lines[i].split()[3]) for i in heads] == [
            int(m) & 0xFF for m in re.findall(r"\{\d+, (\d+), \d+, \d+\}", fir)]


@needs_nvrtc
def test_concurrent_writers_leave_a_valid_entry(tmp_path):
    """Threads of one process compiling the same program at once each write
    through a temporary file of their own; the entry left behind is whole
    (a later process reads it instead of compiling)."""
    import os
    import subprocess
    import sys

    prog = (
        "import sys, threading, numpy as np\n"
        "from simtgo_b200 import tile\n"
        "def work():\n"
        "    g = tile.New()\n"
        "    a = g.Input(np.ones(1000, np.float32))\n"
        "    tile.Sqrt(tile.Add(tile.Abs(a), tile.Scale(a, 3.0))).JITSource(groups=2, compile=True)\n"
        "ts = [threading.Thread(target=work) for _ in range(int(sys.argv[1]))]\n"
        "[t.start() for t in ts]\n"
        "[t.join() for t in ts]\n"
        "print(tile.JITInfo()[2], tile.JITInfo()[4])\n")
    env = dict(os.environ, SIMTGO_B200_CACHE=str(tmp_path / "cache"))
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

    def run(threads):
        out = subprocess.run([sys.executable, "-c", prog, str(threads)], env=env, cwd=root,
                             check=True, capture_output=True, text=True).stdout.split()
        return int(out[0]), int(out[1])

    compiled, hits = run(4)
    assert compiled + hits == 4 and compiled >= 1
    assert run(1) == (0, 1)
    assert not list((tmp_path / "cache").glob("*.tmp*"))
