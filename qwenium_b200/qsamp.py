"""Python host binding of the qsamp C ABI (include/qsamp.h)."""
from __future__ import annotations

import numpy as np

# qsamp_row_params (include/qsamp.h): 48 bytes, naturally aligned.
ROW_PARAMS = np.dtype(
    [
        ("temperature", "<f4"),
        ("top_k", "<i4"),
        ("top_p", "<f4"),
        ("repetition_penalty", "<f4"),
        ("repetition_lookback", "<i4"),
        ("frequency_penalty", "<f4"),
        ("presence_penalty", "<f4"),
        ("softcap", "<f4"),
        ("force_token", "<i4"),
        ("flags", "<i4"),
        ("seed", "<u8"),
    ],
    align=True,
)
