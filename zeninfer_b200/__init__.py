"""zeninfer_b200 -- a B200 (sm_100a) token sampler behind zeninfer's sample.h API.

The compute lives in libzs_sampler.so (zeninfer_b200/csrc, C ABI in
include/zs_sampler.h); this package binds it for Python.
"""

from .sampler import (Rng, SampleResult, Sampler, SamplingParams, argmax_token, rng_seed,
                      sample_token, states_to_tensor, tensor_to_states)

__all__ = ["Rng", "SampleResult", "Sampler", "SamplingParams", "argmax_token", "rng_seed",
           "sample_token", "states_to_tensor", "tensor_to_states"]
