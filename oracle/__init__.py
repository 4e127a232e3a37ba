"""Parity oracle — TEST INFRASTRUCTURE ONLY.

CPU restatements (numpy) of the reference's AR path: ``ar_oracle`` (the decoder) and
``sampler_oracle`` (filters and the draw contract). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / ``--impl reference`` legs
import this package, as the checker or the timed CPU baseline. The CUDA product
(``yue2-mlx_b200/``) never imports, links or executes anything here.
"""
