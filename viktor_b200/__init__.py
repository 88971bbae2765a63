"""B200-native (sm_100a) inference of the Viktor decoder: varlen prefill over projected frames and
CUDA-graph greedy decode behind a drop-in ``DecodeEngine``.  Kernels live in libviktor_b200.so
(C ABI: include/viktor_b200.h), built in-tree by ``python -m viktor_b200.build``."""

from .config import BOS, EOS, PAD, DecoderConfig, KmerTokenizer, get_tokenizer  # noqa: F401
from .decoder import Decoder, KVCache  # noqa: F401
from .engine import DecodeEngine  # noqa: F401
from .model import Basecaller  # noqa: F401
