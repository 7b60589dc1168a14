"""The host oracle of forward-only inference (the reference's src/generate.cpp
set-up and inference::autoregression on the CPU restatement of the runtime
ops), pinned on the CPU: greedy decoding emits the argmax of the logits the
same oracle computes for the padded context, and decoding is reproducible.
The GPU test (tests/test_inference_gpu.py) compares the CUDA runtime with it."""
import numpy as np
import pytest

from oracle import cpu_gpt
from templit_b200 import capi

SEQ = 16

pytestmark = pytest.mark.skipif(not cpu_gpt.available(), reason="oracle GPT library not built")


def config():
    return capi.TlgConfig(family=4, batch=1, seq=SEQ, seed=5, init_std=0.1, lr=3e-4,
                          beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, clip=1.0, world=1,
                          fusion=1, graphs=1, gemm_precision=capi.TL_GEMM_FP32, deferred_wait=0)


@pytest.fixture(scope="module")
def model():
    m = cpu_gpt.OracleGPTInference(config())
    yield m
    m.close()


def test_greedy_token_is_the_logits_argmax(model):
    prompt = [17, 300, 5, 1999, 42]
    eos = 0
    context = np.full(SEQ, eos, np.uint32)  # include/inference.h:66-67
    context[:len(prompt)] = prompt
    logits = model.logits(context)
    first = model.generate(prompt, eos, 1, 1, 1.0, 0)[0]
    assert first == int(np.argmax(logits[len(prompt) - 1]))


def test_decoding_is_reproducible(model):
    prompt = [3, 1, 4, 1, 5, 9]
    a = model.generate(prompt, 0, 11, 40, 0.6, 0)
    b = model.generate(prompt, 0, 11, 40, 0.6, 0)
    assert a == b and len(a) >= 1
