"""The weight registry: device copies of the caller's host weight ranges.

  * draco_b200_register copies a range once; registered bytes grow by the range;
  * a changed weight (inside the sampled words: here the whole tensor is rewritten) is copied
    again on the next call, so outputs follow the new weights;
  * draco_b200_forget drops one range (0 when found, nonzero otherwise) and the next call copies
    it again; draco_b200_reset drops everything; results are unchanged after either.
"""
import ctypes as ct

import numpy as np
import pytest

import dracomancer_llmengine_b200 as dm
from dracomancer_llmengine_b200 import synth

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture()
def reg(dlib):
    dlib.draco_b200_register.argtypes = [ct.c_void_p, ct.c_size_t]
    dlib.draco_b200_forget.argtypes = [ct.c_void_p]
    dlib.draco_b200_registered_bytes.restype = ct.c_size_t
    dlib.draco_b200_reset()
    yield dlib
    dlib.draco_b200_reset()


def test_register_forget_reset(reg, port):
    layer = synth.make_layer(hidden=1024, n_exp=16, n_used=4, inter=256, seed=91)
    X = synth.make_tokens(layer, 6, 92)
    base = reg.draco_b200_registered_bytes()
    gate = layer.gate
    assert reg.draco_b200_register(gate.ctypes.data, gate.nbytes) == 0
    assert reg.draco_b200_registered_bytes() >= base + gate.nbytes
    want = port.layer_forward(layer, X)
    a = dm.forward(layer, X)
    assert rel_l2(a, want) <= 1e-3
    held = reg.draco_b200_registered_bytes()
    assert reg.draco_b200_forget(gate.ctypes.data) == 0
    assert reg.draco_b200_registered_bytes() < held
    assert reg.draco_b200_forget(gate.ctypes.data) != 0     # already gone
    b = dm.forward(layer, X)                                  # copied again on use
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    reg.draco_b200_reset()
    assert reg.draco_b200_registered_bytes() == 0
    c = dm.forward(layer, X)
    assert np.array_equal(a.view(np.uint32), c.view(np.uint32))


def test_changed_weights_are_copied_again(reg, port):
    layer = synth.make_layer(hidden=1024, n_exp=16, n_used=4, inter=256, seed=93)
    X = synth.make_tokens(layer, 5, 94)
    first = dm.forward(layer, X)
    # new expert weights written into the same host buffers
    other = synth.make_layer(hidden=1024, n_exp=16, n_used=4, inter=256, seed=95)
    layer.gate[...] = other.gate
    layer.up[...] = other.up
    layer.down[...] = other.down
    second = dm.forward(layer, X)
    assert not np.array_equal(first, second)
    assert rel_l2(second, port.layer_forward(layer, X)) <= 1e-3
