"""Engine-free online handoff primitives (mirror of ``cachebridge.online``)."""
