"""air_rs.serve."""
