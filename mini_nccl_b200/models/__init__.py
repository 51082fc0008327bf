"""Model families built on this library's ops and parallel layers."""
