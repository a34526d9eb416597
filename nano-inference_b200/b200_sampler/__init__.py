"""B200-native token sampler: a drop-in for nano-inference's ``Sampler``.

``B200Sampler`` keeps the reference's ``SamplerBase.select`` /
``select_batch`` call signature and runs the whole path (penalties,
temperature, top-k, top-p, inverse-CDF draw) in hand-written sm_100a CUDA
kernels behind a C ABI (``include/ns_sampler.h``).  The CUDA library is loaded
on first use; there is no CPU fallback.
"""
from .params import SamplingParams

__all__ = ["SamplingParams", "B200Sampler", "SamplerBase", "VocabParallelSampler"]


def __getattr__(name):
    if name in ("B200Sampler", "SamplerBase"):
        from . import sampler
        return getattr(sampler, name)
    if name == "VocabParallelSampler":
        from . import vocab_parallel
        return vocab_parallel.VocabParallelSampler
    raise AttributeError(name)
