"""CPU backend (epure/kernels/cpu.py in the reference).

The reference binds a Rust fused kernel here (kernel/src/lib.rs) and declines
(returns ``None``) whenever that extension is absent, so the caller
materializes the weight.  This package ships no CPU product kernel: its fused
kernels are the GPU ones.  ``linear`` therefore always declines, which is the
reference's behaviour on an install without the Rust extension, and
``PackedLinear`` then runs ``materialize`` + ``F.linear`` on the CPU.
"""
HAVE_RUST = False


def available():
    return False


def threads():
    return 0


def linear(x, store, cache=None):
    """Always ``None``: the caller falls back to materialize on the CPU."""
    return None
