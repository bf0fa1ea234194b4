"""The Go binding (go/b200/b200.go) against include/simtgo_b200.h, on the CPU.

No Go toolchain exists where this library is built, so the binding cannot
be compiled here; this test holds it to the header instead: every function
the header declares is registered exactly once under its C name, into a
variable whose Go signature has the same parameters, each of the same
width (a pointer of any kind is a pointer: uintptr, unsafe.Pointer or *T),
and the same return; and the Band/Shape structs have the header's fields.
"""
import pathlib
import re

ROOT = pathlib.Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "simtgo_b200.h"
GOFILE = ROOT / "go" / "b200" / "b200.go"

C_SCALARS = {"int32_t": "i32", "int": "i32", "simtgo_tensor": "i32", "int64_t": "i64",
             "uint32_t": "u32", "float": "f32", "double": "f64"}
GO_SCALARS = {"int32": "i32", "int64": "i64", "uint32": "u32", "float32": "f32",
              "float64": "f64", "string": "str", "uintptr": "ptr",
              "unsafe.Pointer": "ptr"}


def c_kind(decl, is_return=False):
    decl = " ".join(decl.replace("const ", " ").split())
    if decl == "void":
        return None
    if "*" in decl or "[" in decl:
        if is_return and decl.replace(" ", "") == "char*":
            return "str"
        return "ptr"
    words = decl.split()
    ty = words[0] if is_return or len(words) == 1 else " ".join(words[:-1])
    return C_SCALARS[ty]


def header_functions():
    s = HEADER.read_text()
    s = re.sub(r"/\*.*?\*/", "", s, flags=re.S)
    s = re.sub(r"#[^\n]*", "", s)
    out = {}
    for ret, name, params in re.findall(r"([A-Za-z_][\w\s\*]*?)\b(simtgo_\w+)\s*\(([^;{]*?)\)\s*;",
                                        s, flags=re.S):
        params = " ".join(params.split())
        kinds = [] if params in ("", "void") else [c_kind(p) for p in params.split(",")]
        out[name] = (c_kind(ret.strip(), True), kinds)
    return out


def go_kind(ty):
    ty = ty.strip()
    if ty.startswith("*"):
        return "ptr"
    return GO_SCALARS[ty]


def go_params(params):
    """Expands Go parameters ("a, b int32, c uintptr") into kinds."""
    kinds, pending = [], 0
    for part in [p.strip() for p in params.split(",") if p.strip()]:
        words = part.split()
        if len(words) == 1:  # a name whose type comes later
            pending += 1
            continue
        k = go_kind(" ".join(words[1:]))
        kinds += [k] * (pending + 1)
        pending = 0
    assert pending == 0, params
    return kinds


def go_bindings():
    src = GOFILE.read_text()
    sigs = {}
    for name, params, ret in re.findall(r"^\s*(\w+)\s+func\(([^)]*)\)\s*([\w.*]*)\s*$", src,
                                        flags=re.M):
        sigs[name] = (go_kind(ret) if ret else None, go_params(params))
    regs = re.findall(r'purego\.RegisterLibFunc\(&(\w+),\s*h,\s*"(\w+)"\)', src)
    return sigs, regs


def test_every_export_is_bound_once_with_matching_widths():
    want = header_functions()
    assert len(want) >= 50, len(want)
    sigs, regs = go_bindings()
    names = [c for _, c in regs]
    assert sorted(set(names)) == sorted(names), "a C function registered twice"
    missing = sorted(set(want) - set(names))
    extra = sorted(set(names) - set(want))
    assert not missing, f"not bound: {missing}"
    assert not extra, f"bound but not in the header: {extra}"
    for var, cname in regs:
        assert var in sigs, f"{cname}: no variable {var}"
        got_ret, got = sigs[var]
        want_ret, wanted = want[cname]
        assert got == wanted, f"{cname} ({var}): Go {got} vs C {wanted}"
        assert got_ret == want_ret, f"{cname} ({var}): returns Go {got_ret} vs C {want_ret}"


def _go_struct(name):
    m = re.search(r"type %s struct \{(.*?)\}" % name, GOFILE.read_text(), flags=re.S)
    assert m, name
    return [go_kind(line.split()[1]) for line in m.group(1).strip().splitlines()]


def test_struct_layouts_match_the_header():
    s = HEADER.read_text()
    assert "typedef struct simtgo_band { float upper; float gain; } simtgo_band;" in s
    assert ("typedef struct simtgo_shape { float floor_gain; int32_t count; double bias; } "
            "simtgo_shape;") in s
    assert _go_struct("Band") == ["f32", "f32"]
    assert _go_struct("Shape") == ["f32", "i32", "f64"]


def test_status_codes_match_the_header():
    s = HEADER.read_text()
    codes = dict((k, int(v)) for k, v in re.findall(r"SIMTGO_(E\w+|OK)\s*=\s*(-?\d+)", s))
    go = GOFILE.read_text()
    names = {"OK": "OK", "ENULL": "ENull", "ELENGTH": "ELength", "EBLOCK": "EBlock",
             "EALIAS": "EAlias", "ELAUNCH": "ELaunch", "ETAPS": "ETaps", "EGRAPH": "EGraph",
             "EDEVICE": "EDevice", "ECOMM": "EComm", "ESIZE": "ESize", "EARG": "EArg"}
    assert set(codes) == set(names)
    for c, g in names.items():
        m = re.search(r"^\s*%s\s+int32\s*=\s*(-?\d+)" % g, go, flags=re.M)
        assert m and int(m.group(1)) == codes[c], (c, g)
