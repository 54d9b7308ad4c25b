"""air_rs.stream."""
