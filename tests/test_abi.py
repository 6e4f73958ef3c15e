"""The C-ABI library loads without a GPU and exports exactly what
include/*.h declares (no compute is called)."""
import ctypes
import glob
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "rustfox_b200", "libfoxcuda.so")


def declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        names |= set(re.findall(r"\b(foxcuda_\w+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    assert {"foxcuda_gemv", "foxcuda_eval", "foxcuda_decode", "foxcuda_model_create"} <= declared()


def test_library_loads_and_exports_every_declared_symbol():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} is missing: build it with `python -m rustfox_b200.build`")
    lib = ctypes.CDLL(LIB)
    missing = [n for n in sorted(declared()) if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (foxcuda_\w+)", out))
    assert declared() <= exported


def test_errors_without_a_device_are_statuses_not_crashes():
    """With no usable GPU the entry points report a status and a message."""
    import rustfox_b200 as rf
    st = rf.lib().foxcuda_init(0)
    if st == 0:
        pytest.skip("a GPU is present")
    assert st in (1, 5, 7) and rf.last_error()
    assert rf.lib().foxcuda_gemv(34, None, None, 1, 256, None, None) == 1
    assert rf.lib().foxcuda_kernel_errors(None) == 7 and rf.last_error()


def test_gemm_argument_checks_run_before_any_device_call():
    """foxcuda_gemm_tq_i8 / _packed reject bad arguments with a status and a
    message before touching the device (host buffers stand in for device
    pointers: only null, size and alignment are looked at)."""
    import rustfox_b200 as rf
    L = rf.lib()
    buf = ctypes.create_string_buffer(1 << 12)
    base = (ctypes.addressof(buf) + 15) // 16 * 16
    p, odd = ctypes.c_void_p(base), ctypes.c_void_p(base + 4)
    cases = [
        (L.foxcuda_gemm_tq_i8(8, p, p, 1, p, 1, 256, p, None), 5),        # Q8_0: no tensor-core pass
        (L.foxcuda_gemm_tq_i8(35, None, p, 1, p, 1, 256, p, None), 1),    # null activations
        (L.foxcuda_gemm_tq_i8(35, p, p, 0, p, 1, 256, p, None), 1),       # no tokens
        (L.foxcuda_gemm_tq_i8(34, p, p, 1, p, 1, 320, p, None), 1),       # K not a multiple of 256
        (L.foxcuda_gemm_tq_i8(35, odd, p, 1, p, 1, 256, p, None), 1),     # unaligned activations
        (L.foxcuda_gemm_tq2_i8_packed(p, p, 1, odd, 1, 256, p, None), 1),  # unaligned weights
        (L.foxcuda_gemm_tq2_i8_packed(p, p, 1, p, 1, 256 * 257, p, None), 1),  # K beyond 65536
    ]
    for got, want in cases:
        assert got == want and rf.last_error()
    assert L.foxcuda_context_set_prefill(None, 1) == 1 and rf.last_error()
    h = ctypes.c_void_p()
    assert L.foxcuda_batch_create(None, 0, ctypes.byref(h)) == 1 and not h.value
    assert L.foxcuda_batch_step(None, None, None) == 1
    assert L.foxcuda_batch_generate(None, None, None, 1, None) == 1
    assert L.foxcuda_context_fill_kv(None, 0, 0) == 1
    assert L.foxcuda_eval_all(None, None, 0, None) == 1
    assert L.foxcuda_context_rewind(None, 0) == 1
    for fn in (L.foxcuda_tp_p2p_clear, L.foxcuda_tp_p2p_pick):
        assert fn(None) == 1
    assert L.foxcuda_tp_p2p_export(None, None) == 1 and L.foxcuda_tp_p2p_open(None, None) == 1
    assert L.foxcuda_tp_p2p_row(None, 0, 0) == 1


def test_struct_layouts_match_the_header(tmp_path):
    """Every public struct of include/foxcuda.h has the size and field
    offsets of its ctypes mirror (compiled with the system C compiler)."""
    import shutil
    from rustfox_b200 import api
    from rustfox_b200.tp import TPShape
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    mirrors = {"foxcuda_model_info": api.ModelInfo, "foxcuda_context_config": api.ContextConfig,
               "foxcuda_sampler_config": api.SamplerConfig, "foxcuda_tp_shape": TPShape}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "foxcuda.h"', "int main(void) {"]
    for cname, py in mirrors.items():
        lines.append(f'printf("{cname} %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname}.{fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c11", "-I", os.path.join(ROOT, "include"), "-o", str(exe), str(src)],
                   check=True)
    got = dict(line.rsplit(" ", 1) for line in subprocess.run(
        [str(exe)], capture_output=True, text=True, check=True).stdout.splitlines())
    for cname, py in mirrors.items():
        assert int(got[cname]) == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert int(got[f"{cname}.{fname}"]) == getattr(py, fname).offset, f"{cname}.{fname}"


def test_ctypes_prototypes_match_the_header():
    """Every bound entry point takes as many arguments as its declaration,
    and a pointer wherever the declaration has one."""
    from rustfox_b200 import api
    text = ""
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text += re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
    decls = {}
    for m in re.finditer(r"\b(foxcuda_\w+)\s*\(([^)]*)\)\s*;", text):
        params = [p.strip() for p in m.group(2).split(",")]
        decls[m.group(1)] = [] if params == ["void"] or params == [""] else params
    assert set(api._PROTOS) <= set(decls), set(api._PROTOS) - set(decls)
    for name, (_, args) in api._PROTOS.items():
        params = decls[name]
        assert len(args) == len(params), f"{name}: {len(args)} bound, {len(params)} declared"
        for a, p in zip(args, params):
            if "*" in p:
                assert a in (ctypes.c_void_p, ctypes.c_char_p) or hasattr(a, "_type_"), f"{name}: {p}"


def test_every_called_entry_point_has_a_prototype():
    """A call without argtypes would pass 64-bit pointers and sizes through
    ctypes' default int conversion: every foxcuda_* the package, the bench
    or the tests call is in the prototype table."""
    from rustfox_b200 import api
    used = set()
    files = glob.glob(os.path.join(ROOT, "rustfox_b200", "*.py")) + glob.glob(os.path.join(ROOT, "tests", "*.py"))
    for f in files + [os.path.join(ROOT, "bench.py"), os.path.join(ROOT, "__graft_entry__.py")]:
        used |= set(re.findall(r"\.(foxcuda_\w+)\s*\(", open(f).read()))
    assert used and not used - set(api._PROTOS), sorted(used - set(api._PROTOS))


def test_python_api_mirrors_upstream_names():
    import rustfox_b200 as rf
    for name in ("gemv", "gemv_tq1_i8", "gemv_tq2_i8", "quantize_activations_i8", "dequant_row",
                 "Model", "Context", "Sampler"):
        assert hasattr(rf, name)
