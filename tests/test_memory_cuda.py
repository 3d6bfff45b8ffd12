"""Memory gate of the reference suite on CUDA (GPU).

Port of the reference's test_18m_train_step_fits_in_16gb
(tests/test_scan.py:259-290 of Anamaya1729/mamba-metal-scan): the
18M-class TinyMamba (d_model 384, 10 layers, d_ff 1536, d_state 8, d_conv 4)
at batch 16 x seq 512, one full train step (forward, backward, AdamW), must
peak below 16 GB. This is the configuration that ran out of memory at 47.7 GB
on the reference's PyTorch scan; the reference measured its peak by polling
the MPS driver from a thread, the CUDA allocator's own peak counter replaces
that here (torch.cuda.max_memory_allocated, reset after a warm-up step).

It runs at the package's default checkpoint stride (8) and at the
reference's (64), which holds 8x fewer checkpoints.
"""
from __future__ import annotations

import pytest
import torch

from mamba_metal import MambaConfig, TinyMamba

pytestmark = pytest.mark.gpu

SEED = 1337
VOCAB = 200            # the reference suite's vocabulary for this gate


def _peak_gb_of_a_train_step(ssm_chunk: int) -> float:
    cfg = MambaConfig(vocab_size=VOCAB, d_model=384, n_layers=10, d_ff=1536, max_seq_len=512,
                      d_state=8, d_conv=4, scan_chunk=128, scan_impl="cuda", ssm_chunk=ssm_chunk)
    torch.manual_seed(SEED)
    model = TinyMamba(cfg).cuda()
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4)
    g = torch.Generator().manual_seed(SEED)
    idx = torch.randint(0, VOCAB, (16, 513), generator=g).cuda()

    def step():
        _, loss = model(idx[:, :-1], idx[:, 1:])
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        return loss

    step()                                     # warm up, allocate everything
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats()
    loss = step()
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() / 2**30
    assert torch.isfinite(loss).item()
    del model, opt
    torch.cuda.empty_cache()
    return peak


@pytest.mark.parametrize("ssm_chunk", [8, 64])
def test_18m_train_step_fits_in_16gb(ssm_chunk):
    gb = _peak_gb_of_a_train_step(ssm_chunk)
    print(f"\n[gate] 18M-class train step, checkpoint stride {ssm_chunk}: peak {gb:.2f} GB "
          "(target < 16 GB)")
    assert gb < 16.0, f"peak {gb:.2f} GB exceeds the 16 GB target"
