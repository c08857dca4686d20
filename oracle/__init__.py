"""CPU oracle for the mixed tile GEMM path (test infrastructure only)."""
