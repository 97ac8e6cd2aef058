"""CPU oracle of the Gemma4.pas sampler (test infrastructure only)."""
