"""The C-ABI library loads on any host and exports what ``include/*.h`` declares.

No kernel runs here: every call below is rejected by host-side validation
before any CUDA work, so these tests need no GPU.
"""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def lib():
    from small_q_attention_b200 import _native, build

    build.build()  # no-op when the in-tree library is up to date
    return _native.library()


def declared_symbols():
    names = []
    for h in (ROOT / "include").glob("*.h"):
        names += re.findall(r"^SQA_API\s+[\w\s\*]+?\b(sqa_\w+)\s*\(", h.read_text(), flags=re.M)
    return sorted(set(names))


def test_header_declares_the_entry_points():
    names = declared_symbols()
    assert {"sqa_forward", "sqa_workspace_bytes", "sqa_merge_partials", "sqa_status_string"} <= set(names)


def test_every_declared_symbol_is_exported(lib):
    from small_q_attention_b200 import _native

    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert set(declared_symbols()) <= set(_native.EXPORTED_SYMBOLS)


def test_abi_version_and_status_strings(lib):
    assert lib.sqa_abi_version() == 110
    for code in range(6):
        assert lib.sqa_status_string(code).decode()
    assert lib.sqa_status_string(99).decode() == "unknown status"


def good_args():
    from small_q_attention_b200._native import SqaArgs

    a = SqaArgs()
    a.query = a.key_cache = a.value_cache = a.block_tables = a.seq_lens = a.out = 256
    a.batch, a.q_len, a.num_q_heads, a.num_kv_heads = 4, 4, 32, 8
    a.head_dim, a.page_size, a.num_pages, a.max_pages = 128, 16, 1024, 512
    return a


@pytest.mark.parametrize("field,value,code", [
    ("head_dim", 64, 2), ("page_size", 32, 2), ("num_q_heads", 16, 2), ("q_len", 17, 2),
    ("q_len", 0, 1), ("num_pages", 0, 1), ("max_pages", 0, 1), ("batch", -1, 1), ("num_ctas", -1, 1),
    ("kernel", 3, 1),
])
def test_forward_rejects_bad_shapes(lib, field, value, code):
    a = good_args()
    setattr(a, field, value)
    assert lib.sqa_forward(ctypes.byref(a), None, 0, None) == code
    st = ctypes.c_int(-1)
    assert lib.sqa_workspace_bytes(ctypes.byref(a), 0, ctypes.byref(st)) == 0
    assert st.value == code


def test_forward_rejects_null_and_misaligned_pointers(lib):
    a = good_args()
    a.query = None
    assert lib.sqa_forward(ctypes.byref(a), None, 0, None) == 1
    a = good_args()
    a.key_cache = 258  # not 16-byte aligned
    assert lib.sqa_forward(ctypes.byref(a), None, 0, None) == 1
    a = good_args()
    a.out_partial = 512  # both output modes at once
    a.out_lse = 1024
    assert lib.sqa_forward(ctypes.byref(a), None, 0, None) == 1
    assert lib.sqa_forward(None, None, 0, None) == 1


def test_merge_rejects_bad_arguments(lib):
    assert lib.sqa_merge_partials(None, None, 2, 10, None, None, None, None) == 1
    assert lib.sqa_merge_partials(256, 256, 0, 10, 256, None, None, None) == 1
    assert lib.sqa_merge_partials(256, 256, 2, 10, None, None, None, None) == 1
    assert lib.sqa_merge_partials(258, 256, 2, 10, 256, None, None, None) == 1


def test_python_layer_maps_codes_to_exceptions():
    from small_q_attention_b200 import _native

    with pytest.raises(ValueError):
        _native.check(2, "x")
    with pytest.raises(RuntimeError):
        _native.check(4, "x")
    _native.check(0, "x")


def test_operator_requires_cuda_without_fallback():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("this host has a GPU")
    from small_q_attention_b200 import small_q_attention

    q = torch.zeros(1, 2, 32, 128, dtype=torch.float16)
    cache = torch.zeros(4, 16, 8, 128, dtype=torch.float16)
    with pytest.raises(RuntimeError):
        small_q_attention(q, cache, cache, torch.zeros(1, 4, dtype=torch.int32),
                          torch.tensor([32], dtype=torch.int32), 16)


def test_struct_layouts_match_the_header(tmp_path):
    """The ctypes mirrors have the C structs' size and every field offset."""
    import ctypes
    import shutil
    import subprocess

    from small_q_attention_b200._native import SqaAppendArgs, SqaArgs

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    include = Path(__file__).resolve().parents[1] / "include"
    lines = ["#include <stddef.h>", "#include <stdio.h>", '#include "small_q_attention.h"', "int main(void) {"]
    for cls, cname in ((SqaArgs, "sqa_args"), (SqaAppendArgs, "sqa_append_args")):
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for name, _ in cls._fields_:
            lines.append(f'  printf("{cname} {name} %zu\\n", offsetof({cname}, {name}));')
    lines.append("  return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(include), str(src), "-o", str(exe)], check=True)
    got = dict(((a, b), int(c)) for a, b, c in (ln.split() for ln in subprocess.run(
        [str(exe)], check=True, capture_output=True, text=True).stdout.splitlines()))
    for cls, cname in ((SqaArgs, "sqa_args"), (SqaAppendArgs, "sqa_append_args")):
        assert got[(cname, "size")] == ctypes.sizeof(cls)
        for name, _ in cls._fields_:
            assert got[(cname, name)] == getattr(cls, name).offset, (cname, name)


def test_torch_extension_registers_the_operators():
    """The torch extension loads without a GPU, registers torch.ops.sqa_b200.*, and
    its Meta kernels give the output shapes (what torch.compile traces with); a
    CPU tensor is rejected with the upstream's ValueError before any launch."""
    import torch

    from small_q_attention_b200 import _native, build

    build.build_torch_ext()  # no-op when up to date
    ext = _native.torch_ext()
    assert ext.abi_version() == 110
    q = torch.empty(2, 4, 32, 128, dtype=torch.float16, device="meta")
    k = torch.empty(64, 16, 8, 128, dtype=torch.float16, device="meta")
    bt = torch.empty(2, 32, dtype=torch.int32, device="meta")
    sl = torch.empty(2, dtype=torch.int32, device="meta")
    out = torch.ops.sqa_b200.small_q_attention(q, k, k, bt, sl, 16)
    assert out.shape == q.shape and out.dtype == torch.float16
    o, lse = torch.ops.sqa_b200.small_q_attention_partial(q, k, k, bt, sl, 16, mask_lens=sl)
    assert o.shape == q.shape and o.dtype == torch.float32 and lse.shape == (2, 4, 32)
    cpu = [torch.zeros(2, 4, 32, 128, dtype=torch.float16), torch.zeros(64, 16, 8, 128, dtype=torch.float16)]
    with pytest.raises(ValueError, match="CUDA tensors"):
        ext.forward(cpu[0], cpu[1], cpu[1], torch.zeros(2, 32, dtype=torch.int32),
                    torch.zeros(2, dtype=torch.int32), 16, 0, None, None, 0, 0, 0, False, 0, 0.0, 1.0, 0, 0)


def test_torch_extension_shares_the_process_cpp_runtime():
    """The extension must link the shared libstdc++ that torch uses, not carry a
    private static copy: its C++ exceptions are caught and rethrown by torch's
    error translation, which is undefined behaviour across two runtimes."""
    import shutil
    import subprocess

    from small_q_attention_b200 import build

    if not (shutil.which("readelf") and shutil.which("nm")):
        pytest.skip("binutils not available")
    path = build.build_torch_ext()
    needed = subprocess.run(["readelf", "-d", str(path)], capture_output=True, text=True).stdout
    assert "libstdc++.so.6" in needed
    exported = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True).stdout
    assert "__cxa_allocate_exception" not in exported and "__cxa_throw" not in exported


def test_extension_loads_first_in_a_fresh_process():
    """A process whose first call is the operator loads the torch extension before
    the C library: that must not deadlock (a fresh interpreter, bounded)."""
    import subprocess
    import sys

    code = ("import sys; sys.path.insert(0, %r)\n"
            "from small_q_attention_b200 import _native\n"
            "ext = _native.torch_ext()\n"
            "assert ext.abi_version() == _native.library().sqa_abi_version()\n"
            "print('ok')\n") % str(ROOT)
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0 and res.stdout.strip().endswith("ok"), res.stderr[-2000:]
