"""CPU oracle for the gpt-oss MoE layer — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic that hareramray/BlockStreamer
runs for its gpt-oss mixture-of-experts layer, so that the CUDA path can be
checked against it. It is the checker, never the thing measured or shipped:
only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it. The product package
``blockstreamer_b200`` never imports anything from here and fails loudly when
its CUDA library is missing.

Modules
-------
``oracle.mxfp4``  bit-exact MXFP4 -> bf16/fp32 dequant (numpy), restating
                  ``transformers.integrations.mxfp4._convert_moe_packed_tensors``
                  (transformers 5.5.0, integrations/mxfp4.py:279-330) as called by
                  ``block_streamer/gptoss.py:24-42``.
``oracle.moe``    the router (transformers models/gpt_oss/modeling_gpt_oss.py:117-130),
                  the expert loop (``block_streamer/gptoss.py:130-177``) in the
                  reference's own bf16 rounding order ("port"), and the same math
                  evaluated in fp32 (the accuracy target).

Pinning: ``tests/golden/make_golden.py`` runs the reference itself (importable
in the development container) and commits its outputs under ``tests/golden``;
``tests/test_oracle.py`` checks this oracle against those fixtures.
"""
