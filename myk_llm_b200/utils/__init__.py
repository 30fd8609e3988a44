"""Small shared helpers (sweep planning / running for the research testbeds)."""
