---------------------------- MODULE HostLaneReuseN ----------------------------
(* One range staged through pinned-host lanes. Piece k uses lane            *)
(* (k-1) % Lanes. Each of S source ranks copies its part of piece k into    *)
(* its bounce buffer of that lane (D2H, in order per source and lane, and   *)
(* -- unless SkipReuseWait -- only after every H2D of piece k-Lanes         *)
(* finished: LaneFree). When S > 1 the host folds the S bounce buffers      *)
(* into the lane's output (in order per lane); every one of D destination   *)
(* ranks then copies the output (or, for S = 1, the source's bounce) into   *)
(* its buffer (H2D, in order per destination and lane). A fold reads piece  *)
(* k only if every bounce still holds piece k; otherwise it yields -1.      *)
EXTENDS Integers, FiniteSets

CONSTANTS Pieces, Lanes, S, D, SkipReuseWait
VARIABLES produced, folded, consumed, bounce, out, output
vars == <<produced, folded, consumed, bounce, out, output>>

Chunks == 1..Pieces
Sources == 0..(S - 1)
Dests == 0..(D - 1)
LaneOf(k) == (k - 1) % Lanes
Fold == S > 1

Init == /\ produced = {} /\ folded = {} /\ consumed = {}
        /\ bounce = [q \in Sources |-> [l \in 0..(Lanes - 1) |-> 0]]
        /\ out = [l \in 0..(Lanes - 1) |-> 0]
        /\ output = [k \in Chunks |-> [r \in Dests |-> 0]]

LaneFree(k) == k <= Lanes \/ \A r \in Dests : <<k - Lanes, r>> \in consumed

Produce(k, q) ==
  /\ <<k, q>> \notin produced
  /\ (k <= Lanes \/ <<k - Lanes, q>> \in produced)
  /\ (SkipReuseWait \/ LaneFree(k))
  /\ bounce' = [bounce EXCEPT ![q][LaneOf(k)] = k]
  /\ produced' = produced \cup {<<k, q>>}
  /\ UNCHANGED <<folded, consumed, out, output>>

HostFold(k) ==
  /\ Fold /\ k \notin folded
  /\ \A q \in Sources : <<k, q>> \in produced
  /\ (k <= Lanes \/ (k - Lanes) \in folded)
  /\ out' = [out EXCEPT ![LaneOf(k)] =
               IF \A q \in Sources : bounce[q][LaneOf(k)] = k THEN k ELSE 0 - 1]
  /\ folded' = folded \cup {k}
  /\ UNCHANGED <<produced, consumed, bounce, output>>

Consume(k, r) ==
  /\ <<k, r>> \notin consumed
  /\ IF Fold THEN k \in folded ELSE \A q \in Sources : <<k, q>> \in produced
  /\ (k <= Lanes \/ <<k - Lanes, r>> \in consumed)
  /\ output' = [output EXCEPT ![k][r] = IF Fold THEN out[LaneOf(k)] ELSE bounce[0][LaneOf(k)]]
  /\ consumed' = consumed \cup {<<k, r>>}
  /\ UNCHANGED <<produced, folded, bounce, out>>

Next == \/ \E k \in Chunks, q \in Sources : Produce(k, q)
        \/ \E k \in Chunks : HostFold(k)
        \/ \E k \in Chunks, r \in Dests : Consume(k, r)
Spec == Init /\ [][Next]_vars

CorrectOutputs == \A c \in consumed : output[c[1]][c[2]] = c[1]
ProducedBeforeConsumed == \A c \in consumed : \A q \in Sources : <<c[1], q>> \in produced
===============================================================================
