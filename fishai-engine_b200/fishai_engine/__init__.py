"""fishai_engine — B200 (sm_100a) implementation of the fishai-engine token
loop behind the crate's model API (gguf, quant, model, kv_cache, sampling).

Mirrors the reference crate's modules (src/lib.rs:14-33); every compute call
goes through the CUDA library lib/libfishai_cuda.so."""
from ._lib import FishaiError, build  # noqa: F401
from .gguf import GGUFFile  # noqa: F401
from .kv_cache import KVCache  # noqa: F401
from .model import GenerationConfig, GenerationState, ModelConfig, ModelWeights  # noqa: F401
from .sampling import Sampler, SamplerConfig  # noqa: F401
