"""B200-native drop-in for the reference's `flash_evict` package.

`prefill`, `evict` and `select_tokens` keep the reference's signatures
(flash_evict/__init__.py:1-3 of the reference); the compute runs in the
sm_100a native library bound by `_lib`.  `gather_tokens`,
`select_and_gather` and `evict_compact` (flash_evict.compact) add the KV
compaction the reference's adapters perform after selection;
`check_status` reports failures of kernels launched by earlier calls.
"""
from .prefill import prefill, evict, select_tokens
from .compact import gather_tokens, select_and_gather, evict_compact
from .status import check_status

__all__ = ["prefill", "evict", "select_tokens", "gather_tokens", "select_and_gather", "evict_compact", "check_status"]
