"""An encoder through the drop-in boundary: a synthetic EmbeddingGemma 2 file
(`gemma-embedding2`) read by the reference's GGUF reader and description,
planned with its encoder working set, uploaded by its routes and piece
writer, and its encoder graph (src/core/graph/encoder.cpp, the
architecture's EncodeFn) built and run by the CUDA Program
(integration/libcharlotte_program.so): the norm's encoder forms, rope's
encode form, block attention's two launches as one, the GatedByInput
product, mean pooling and the unit-length vector read back.

Parity tier: bit-exact — the embedding equals the oracle's pass over the
same weights in the reference's order (tests/encoder_model.py), for steps
longer and shorter than the sliding layers' window, and a second step on
the same program gives its own bits."""
import ctypes
import os

import numpy as np
import pytest

import encoder_model as E
from test_program_gpu import Harness

pytestmark = pytest.mark.gpu


class EncoderHarness(Harness):
    def __init__(self, path):
        super().__init__(path)
        self.L.cbh_embedding_length.restype = ctypes.c_uint32
        self.L.cbh_embedding_length.argtypes = [ctypes.c_void_p]
        self.L.cbh_embedding.restype = ctypes.c_int
        self.L.cbh_embedding.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        self.length = self.L.cbh_embedding_length(self.h)

    def embed(self, ids):
        self.step(ids, 0, logits=True)
        out = np.empty(self.length, np.float32)
        assert self.L.cbh_embedding(self.h, out.ctypes.data) == 0
        return out


@pytest.fixture(scope="module")
def encoder(tmp_path_factory):
    m = E.synthesize(E.EncoderArch(), seed=3)
    path = str(tmp_path_factory.mktemp("enc") / "embedding_gemma2.gguf")
    E.write_gguf(m, path)
    h = EncoderHarness(path)
    yield m, h
    h.L.cbh_close(h.h)


@pytest.mark.parametrize("tokens", [100, 7])
def test_embedding_bit_exact(cuda, encoder, tokens):
    m, h = encoder
    assert h.length == m["arch"].embedding
    ids = np.random.default_rng(tokens).integers(0, m["arch"].vocab, tokens).astype(np.uint32)
    got = h.embed(ids)
    want = E.oracle_embedding(m, ids)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
    assert abs(float(np.linalg.norm(got.astype(np.float64))) - 1.0) < 1e-5


def test_embedding_of_one_token(cuda, encoder):
    m, h = encoder
    got = h.embed([5])
    np.testing.assert_array_equal(got.view(np.uint32), E.oracle_embedding(m, [5]).view(np.uint32))
