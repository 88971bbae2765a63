"""CPU oracle for the Viktor decoder hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / ``--impl reference``
legs may import this package.  The product path (``viktor_b200``) never routes through it.
"""

from .decoder_np import (BOS, EOS, PAD, OracleConfig, OracleModel, OracleTokenizer, apply_rope,  # noqa: F401
                         bases_emitted, rms_norm, rope_tables)
