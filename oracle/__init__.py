"""CPU oracle for the Oasis-500M DiT denoising forward — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the algorithms of the hot path that the
B200 library replaces.  It exists to check the CUDA path, never to stand in
for it: only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` leg / ``--impl reference`` arm may import it.  The product
package must never import anything from here.

Contents
--------
``dit_ref``      PyTorch fp32 restatement of the open-oasis ``DiT-S/2`` forward
                 (the third-party module the reference imports at
                 ``worldserve/models/oasis.py:66-77``).  Upstream open-oasis is
                 cloned unpinned by the reference (``benchmarks/common.py:45-55``)
                 and is absent here, so DiT-forward parity with upstream is
                 *unpinned*; the temporal-attention sub-module is pinned against
                 the reference's own restatement
                 (``kv_cache/oasis_temporal_persistent_wrapper.py:86-150``).
``quant_ref``    numpy restatement of ``ProgressiveKVQuantizer.quantize_to_fp8`` /
                 ``quantize_to_int4`` / dequantisers
                 (``kv_cache/progressive_quant.py:113-257``), pinned bit-exactly
                 against fixtures generated from the reference itself.
``sampler_ref``  numpy restatement of the DDIM v-step (``models/oasis.py:218-228``),
                 the DPM-Solver++ 2M v-step (``benchmarks/optimised/
                 oasis_dpmpp_modal.py:143-164``), the Adams–Bashforth
                 ``DPMSolverPPSampler.step`` (``samplers/dpm_solver_pp.py:85-143``)
                 and the sigmoid beta schedule; pinned against fixtures from the
                 reference's importable code.
"""
