"""The TensorFlow op surface (tf_op/) compiled without TensorFlow and driven as TF would.

tf_op/sdpa_ops.cc and tf_op/sdpa_kernels.cc are compiled against the mock TF
headers of oracle/tf_shim/ and linked with libsdpa_b200.so; the kernels they
register are then run through the same driver that runs the reference's own
kernels (oracle/ref_wrap.cc).  CPU: registrations, op definitions, every
validation message.  GPU: full Sdpa / SdpaGrad vs the library's own API.
"""
import ctypes
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tf-custom-flash-attention_b200")
OUT = os.path.join(ROOT, "tests", "_build", "libtfop_shim.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def build():
    srcs = [os.path.join(PKG, "tf_op", "sdpa_ops.cc"), os.path.join(PKG, "tf_op", "sdpa_kernels.cc"),
            os.path.join(ROOT, "oracle", "ref_wrap.cc")]
    if os.path.exists(OUT) and all(os.path.getmtime(s) <= os.path.getmtime(OUT) for s in srcs):
        return OUT
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = ["g++", "-std=c++17", "-O1", "-fPIC", "-shared", "-DGOOGLE_CUDA=1", "-DTFS_WITH_CUDA_RUNTIME",
           "-I" + os.path.join(ROOT, "oracle", "tf_shim"), "-I" + os.path.join(ROOT, "oracle"),
           "-I" + os.path.join(CUDA, "include"), *srcs, "-o", OUT, "-L" + PKG, "-lsdpa_b200",
           "-Wl,-rpath," + PKG, "-L" + os.path.join(CUDA, "lib64"), "-lcudart", "-lpthread"]
    subprocess.run(cmd, check=True)
    return OUT


@pytest.fixture(scope="module")
def tfop():
    return ctypes.CDLL(build())


def _driver(lib):
    """oracle.ref's ctypes plumbing pointed at this library (its ref_run drives any registry)."""
    from oracle import ref

    lib.ref_run.restype = ctypes.c_int
    lib.ref_run.argtypes = [
        ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
        ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_long), ctypes.POINTER(ctypes.c_long),
        ctypes.c_int, ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_long),
        ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int,
    ]
    lib.ref_set_num_threads.argtypes = [ctypes.c_int]
    lib.ref_get_num_threads.restype = ctypes.c_int
    lib.ref_num_kernels.restype = ctypes.c_int
    lib.ref_kernel_info.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                    ctypes.POINTER(ctypes.c_int)]
    ref._libs["libsdpa_ref_gpu.so"] = lib
    ref._libs["libsdpa_ref_cpu.so"] = lib
    return ref


def test_registrations(tfop):
    ref = _driver(tfop)
    ks = sorted(ref.registered_kernels("GPU"))
    assert ks == sorted([("Sdpa", "GPU", 1), ("Sdpa", "GPU", 19), ("SdpaGrad", "GPU", 1), ("SdpaGrad", "GPU", 19)])


def test_validation_messages_match_reference(tfop):
    ref = _driver(tfop)
    f = np.float32
    q = np.zeros((2, 8, 16), f)
    k = np.zeros((2, 8, 16), f)
    v = np.zeros((2, 8, 4), f)
    cases = [
        ((q, k[:1].copy(), v), {}, "K batch size mismatch"),
        ((q, k[:, :, :8].copy(), v), {}, "K feature size mismatch"),
        ((q, k, v[:1].copy()), {}, "V batch size mismatch"),
        ((q, k, v[:, :4].copy()), {}, "V seq size mismatch"),
        ((q, k[:, :4].copy(), v[:, :4].copy()), {"causal_mask": True}, "seq size Q != K while causal_mask = True"),
        ((np.zeros((2, 8, 130), f), np.zeros((2, 8, 130), f), v), {},
         "CUDA kernel does not support feature size over 128. Set smaller feature size or use more heads"),
    ]
    for args, kw, msg in cases:
        with pytest.raises(ref.RefOpError) as e:
            ref.ref_sdpa(*args, 1, 2, device="GPU", **kw)
        assert str(e.value) == msg
    o = np.zeros((2, 8, 4), f)
    s = np.zeros((2, 8), f)
    for bad, msg in [((o[:1].copy(), s, o), "O batch size mismatch"), ((o, s, o[:, :7].copy()), "dO seq size mismatch"),
                     ((o, s[:, :3].copy(), o), "S seq size mismatch")]:
        with pytest.raises(ref.RefOpError) as e:
            ref.ref_sdpa_grad(q, k, v, bad[0], bad[1], bad[2], 1, 2, device="GPU")
        assert str(e.value) == msg


@pytest.mark.gpu
@pytest.mark.parametrize("dt", ["float16", "float32"])
def test_tf_surface_runs_the_kernels(tfop, dt):
    import importlib

    import torch

    ref = _driver(tfop)
    fa = importlib.import_module("tf-custom-flash-attention_b200")
    tdt = getattr(torch, dt)
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v, do = (torch.randn(2, 256, 64, generator=g, device="cuda").to(tdt) for _ in range(4))
    kw = dict(scale=0.125, dropout=0.1, causal_mask=True)
    o1, s1 = ref.ref_sdpa(q, k, v, 5, 9, device="GPU", **kw)
    g1 = ref.ref_sdpa_grad(q, k, v, o1, s1, do, 5, 9, device="GPU", **kw)
    o2, s2 = fa.sdpa(q, k, v, 5, 9, **kw)
    g2 = fa.sdpa_grad(q, k, v, o2, s2, do, 5, 9, **kw)
    torch.cuda.synchronize()
    for a, b in zip((o1, s1, *g1), (o2, s2, *g2)):
        assert torch.equal(a, b)
