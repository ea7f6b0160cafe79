"""CPU checks of the drop-in boundary: the C-ABI library loads and exports
every symbol include/mask_loss_b200.h declares, the host-only entries answer,
and the Python surfaces mirror the reference's names and reject bad input.
No kernel is launched here."""
import ctypes
import os
import re

import pytest
import torch

import mask_loss_b200
from mask_loss_b200 import _lib, ops
from mask_loss_b200 import functions as F

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "mask_loss_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(ml_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = header_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), n
    assert sorted(_lib.SIGNATURES) == names


def test_host_only_entries():
    lib = _lib.load()
    assert lib.ml_version() >= 100
    assert lib.ml_status_string(0) == b"ok"
    assert lib.ml_gt_out(10, 0) == 9
    assert lib.ml_gt_out(10, -1) == 10
    assert lib.ml_gt_out(10, 10) == 10
    d = _lib.Dims(1, 16, 100, 256, 256, 256, 256, 134, 31)
    p = ops._params(background_index=0, uncertainty_gamma=0.0)
    n = lib.ml_mask_matching_workspace_size(ctypes.byref(d), ctypes.byref(p))
    assert 0 < n < 64 << 20
    bad = _lib.Dims(1, 2, 3, 5, 5, 12, 12, 4, 3)  # 12 not a multiple of 5
    assert lib.ml_mask_matching_workspace_size(ctypes.byref(bad), ctypes.byref(p)) == 0
    assert b"integer multiple" in lib.ml_last_error()


def _header_struct_fields(name):
    src = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (name, name), src, flags=re.S).group(1)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if decl:
            fields += [f.strip() for f in re.sub(r"^\w+\s+", "", decl).split(",")]
    return fields


def test_ctypes_structs_mirror_the_header():
    # field names in declaration order; the C layout rules then give both
    # sides the same offsets and size
    assert [f[0] for f in _lib.Params._fields_] == _header_struct_fields("ml_params")
    assert [f[0] for f in _lib.Dims._fields_] == _header_struct_fields("ml_dims")


def test_logits_dtype_is_validated_before_any_device_work():
    lib = _lib.load()
    d = _lib.Dims(1, 1, 4, 8, 8, 8, 8, 5, 3)
    p = ops._params(background_index=0, uncertainty_gamma=0.0)
    p.logits_dtype = 3
    rc = lib.ml_pairwise_mask_loss_forward(ctypes.byref(d), ctypes.byref(p), None, None, None,
                                           None, None, None, 0, None)
    assert rc == 1  # ML_EINVAL
    assert b"logits_dtype" in lib.ml_last_error()


def test_op_surface_names():
    # src/bindings.cpp:157-169
    for name in ["forward_sigmoid_ce_loss", "backward_sigmoid_ce_loss", "forward_pw_sigmoid_ce_loss",
                 "forward_dice_loss", "backward_dice_loss", "forward_pw_dice_loss",
                 "pairwise_mask_loss_forward", "mask_matching", "mask_matching_backward",
                 "forward_pw_sigmoid_label_loss", "forward_pw_softmax_label_loss"]:
        assert callable(getattr(ops, name)), name
    for name in ["MaskMatchingFunction", "PairwiseMaskLossFunction", "PairwiseSigmoidCELossFunction",
                 "PairwiseDiceLossFunction", "PairwiseSigmoidLabelLossFunction",
                 "PairwiseSoftmaxLabelLossFunction", "pairwise_softmax_label_loss",
                 "SigmoidCELossFunction", "DiceLossFunction"]:
        assert hasattr(F, name), name


def _cpu_inputs():
    ml = torch.zeros(1, 2, 4, 8, 8)
    mt = torch.zeros(2, 8, 8, dtype=torch.long)
    cl = torch.zeros(1, 2, 4, 5)
    ct = torch.full((2, 3), -1, dtype=torch.long)
    return ml, mt, cl, ct


def test_ops_reject_cpu_tensors():
    ml, mt, cl, ct = _cpu_inputs()
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        ops.mask_matching(ml, mt, cl, ct, 1.0)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        ops.pairwise_mask_loss_forward(ml, mt, cl, ct, 1.0)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        ops.forward_pw_softmax_label_loss(cl, ct)


def test_function_argument_validation():
    ml, mt, cl, ct = _cpu_inputs()
    base = [ml, mt, cl, ct, 1.0, 1.0, 1.0, 1.0, 0, 1.0, 0.05, True, 1e30, None, False, False, 1,
            "global", 0.0, None, None, None]
    bad = list(base); bad[17] = "hungary"
    with pytest.raises(ValueError, match="Unknown assignment_strategy"):
        F.MaskMatchingFunction.apply(*bad)
    bad = list(base); bad[16] = -1
    with pytest.raises(ValueError, match="K must be non-negative"):
        F.MaskMatchingFunction.apply(*bad)
    bad = list(base); bad[9] = -0.5
    with pytest.raises(ValueError, match="uncertainty_gamma must be non-negative"):
        F.MaskMatchingFunction.apply(*bad)
    with pytest.raises(ValueError, match="void_class_index must be provided"):
        F.MaskMatchingFunction.apply(*(base[:14] + [True] + base[15:]), None, "softmax")
    with pytest.raises(ValueError, match="incorrect void index"):
        F.MaskMatchingFunction.apply(*base, 9, "softmax")
    with pytest.raises(ValueError, match="label_loss"):
        F.MaskMatchingFunction.apply(*base, None, "hinge")


def test_semantic_losses_reject_cpu_tensors():
    """The semantic ops run on the GPU only (no CPU fallback)."""
    import torch
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.forward_sigmoid_ce_loss(torch.zeros(1, 1, 2, 4, 4), torch.zeros(1, 4, 4, dtype=torch.long), 1.0)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.forward_dice_loss(torch.zeros(1, 1, 2, 4, 4), torch.zeros(1, 4, 4, dtype=torch.long), 1.0, 1.0)


def test_header_compiles_as_c_and_links(tmp_path):
    # a plain C99 caller: the header is valid C, the library links, the
    # host-only entries answer, and the struct sizes equal the ctypes mirrors
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("no C compiler")
    libdir = os.path.dirname(_lib.load()._name)
    src = tmp_path / "caller.c"
    src.write_text(
        '#include "mask_loss_b200.h"\n#include <stdio.h>\n'
        "int main(void) {\n"
        "  ml_dims d = {1, 2, 3, 8, 8, 8, 8, 5, 3};\n"
        "  ml_params p = {0};\n"
        "  size_t n = ml_mask_matching_workspace_size(&d, &p);\n"
        '  printf("%d %zu %zu %zu\\n", ml_version(), n, sizeof(ml_params), sizeof(ml_dims));\n'
        "  return 0;\n}\n")
    exe = tmp_path / "caller"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-pedantic",
                    "-I" + os.path.join(REPO, "include"), str(src), "-L" + libdir,
                    "-lmask_loss_b200", "-Wl,-rpath," + libdir, "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert int(out[0]) == _lib.load().ml_version()
    assert int(out[1]) > 0
    assert int(out[2]) == ctypes.sizeof(_lib.Params)
    assert int(out[3]) == ctypes.sizeof(_lib.Dims)
