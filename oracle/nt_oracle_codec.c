/* codec: filled in below */
