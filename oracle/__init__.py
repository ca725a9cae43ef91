"""CPU oracle for the streaming listener step -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the reference algorithm of the listener
hot path so that the CUDA implementation can be checked against it:

- ``mel_ref``        : incremental 80 ms log-mel extraction
                       (duplex_kernel/listener.py:1807-1850, with
                       transformers 5.5.0 Gemma4AudioFeatureExtractor
                       window/filterbank, feature_extraction_gemma4.py:95-160)
- ``conformer_ref``  : exact streaming Q2 step of the Gemma 4 audio Conformer
                       (duplex_kernel/streaming_conformer.py:700-888 over the
                       transformers modules models/gemma4/modeling_gemma4.py)
- ``film_ref``       : FrameResidualQueryFiLMAdapter residual
                       (duplex_kernel/frame_residual_adapter.py:156-237)
- ``packer_ref``     : tick snapshot order, coordinator head ordering and the
                       persistent slot policy (shared_listener_scheduler.py:486-535,
                       listener_microbatch.py:170-279, streaming_conformer.py:571-615,
                       904-967)

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package, and only as
the checker or the timed CPU baseline.  The product path never imports it.

Parity pinning: every module is checked against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py`` imports the
reference classes in the build container); see ``tests/test_oracle_golden.py``.
"""
