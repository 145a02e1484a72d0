"""Backend plumbing kept API-compatible with the reference's `fast_trimul.core`:
the plug-in registry, the input guard, the dispatcher and the scoped backend
preference (fast_trimul/core/{registry,context,dispatch,decorators}.py)."""
