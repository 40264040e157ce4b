"""Operation declaration (TEMPO-OP), oracle arithmetic and coverage."""
