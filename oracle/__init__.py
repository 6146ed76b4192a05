"""CPU oracle for the DeltaPhase inference hot path (TEST INFRASTRUCTURE ONLY).

This package restates, in numpy, the algorithms of the reference implementation
(mcarbonell/delta-phase v1.3.0) for the paths that the CUDA library replaces:

* ``oracle.core``    -- chunkwise complex delta rule, its token recurrence, the
                        decode step and the phasor Gram
                        (delta_phase/kernels/triton_chunk_delta.py,
                        delta_phase/layers.py).
* ``oracle.laplace`` -- LaplacePhaseCore chunkwise solve and its token loop
                        (delta_phase/layers.py).
* ``oracle.spectral``-- Hadamard / DCT-II / "Haar" matrices and the spectral
                        Lerp FFN (delta_phase/spectral.py, delta_phase/layers.py).
* ``oracle.block``   -- the block glue (LayerNorm, causal conv, projections) around
                        the core, for block forward/step parity.

Every function cites the reference file:line it follows.  The oracle is pinned
against golden vectors produced by the reference itself (tests/golden/, made by
tests/golden/make_golden.py).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline arm
may import this package, and only as the checker / the timed CPU port.  The
product package ``delta_phase_b200`` never imports it.
"""
