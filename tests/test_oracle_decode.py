"""The oracle's paged_decode_attention (out and lse) against the reference's
paged_decode_attention_ref run on the same cases (tests/golden/decode.npz)."""
import numpy as np
import torch

import cases
from oracle import actkv_oracle as O


def test_oracle_decode_matches_reference_golden(golden):
    g = golden("decode.npz")
    for c, spec in enumerate(g["meta"]["cases"]):
        case = cases.build_sessions(**spec)
        assert cases.digest(case.kv) == str(g[f"kv_sha_{c}"])
        q = torch.cat([qq[0] for qq in case.q], 0).float().numpy()
        out, lse = O.paged_decode_attention(q, cases.to_np(case.kv)[0],
                                            cases.block_table_array(case.tables).astype(np.int64), case.seq_lens)
        np.testing.assert_allclose(lse, g[f"lse_{c}"], rtol=1e-6, atol=2e-6)
        np.testing.assert_allclose(out, g[f"out_{c}"], rtol=1e-5, atol=2e-6)
