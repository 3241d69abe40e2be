"""CPU oracle for the Prometheus fp32 compute path (test infrastructure only)."""
